// Helpers shared by the translation units of libb2attn.so (not part of the
// C ABI): the per-thread error message read by b2_last_error().
#pragma once

#include <stdint.h>

int b2_record_error(int code, const char *message);  // stores the message, returns code
int b2_clear_error();                                // clears the message, returns B2_OK
uint64_t b2_wait_limit_ns();                          // the current limit of a wait on another thread
