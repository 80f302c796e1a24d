"""The minimal ctypes binding a maintainer of the reference's Python decode
loop adds to call libb2attn.so directly (the reference drives its NPU
operators from Python, e.g. experiments/007_lfm25_npu_chat.py:160-196).

It is self-contained on purpose: no torch and no other module of this
package, only the shared library and device pointers from any allocator.
The package's own binding (_lib.py) declares the same argument types for
every entry point; tests/test_abi_cpu.py keeps the two in step.

    lib = bind("ryzenai-npu-lab_b200/libb2attn.so")
    rc = lib.b2_decode_step(qkv_ptr, 2048, gq_ptr, gk_ptr, F32(1e-5), cos_ptr, sin_ptr, rows,
                            past_ptr, None, tables_ptr, max_blocks, kpool_ptr, vpool_ptr,
                            num_blocks, batch, bps, F32(0.125), 1 | 2 | 4, ctx_ptr, None,
                            None, None, ml_ptr, o_ptr, counters_ptr, 0, err_ptr, stream)
    if rc:
        raise RuntimeError(last_error(lib))
"""
import ctypes

P, I32, I64, F32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float

# entry point -> argument types, in the order of include/b2_decode_attn.h
ARGTYPES = {
    # q/k norm + RoPE + KV append (append_attention_cache + norm_rope)
    "b2_append_rope": [P, I64, P, P, F32, P, P, I32, P, P, I32, P, P, I32, P, I32, I32, P, P],
    # split-KV decode into partial states (attention_context*)
    "b2_decode_attn": [P, P, P, I32, P, I32, P, I32, I32, I32, F32, P, P, P, P],
    # log-sum-exp merge of the partial states
    "b2_combine": [P, P, I32, P, I32, I32, P, P, P, P],
    # the three above in one persistent launch (the default path)
    "b2_decode_step_counters": [I32],
    "b2_decode_step": [P, I64, P, P, F32, P, P, I32, P, P, P, I32, P, P, I32,
                       I32, I32, F32, I32, P, P, P, P, P, P, P, I32, P, P],
    # limits of the kernels' bounded waits (the watchdog of a run)
    "b2_set_wait_limits": [I64, I64],
    "b2_last_error": [ctypes.c_char_p, ctypes.c_int],
}


def bind(path: str) -> ctypes.CDLL:
    """Load the library and declare the entry points above (every one
    returns int: 0 or a negative status)."""
    lib = ctypes.CDLL(path)
    for name, args in ARGTYPES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    return lib


def last_error(lib: ctypes.CDLL) -> str:
    """The calling thread's last error message."""
    buf = ctypes.create_string_buffer(512)
    lib.b2_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")
