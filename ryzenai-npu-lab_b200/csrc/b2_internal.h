// Helpers shared by the translation units of libb2attn.so (not part of the
// C ABI): the per-thread error message read by b2_last_error().
#pragma once

int b2_record_error(int code, const char *message);  // stores the message, returns code
int b2_clear_error();                                // clears the message, returns B2_OK
