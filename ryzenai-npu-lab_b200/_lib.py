"""ctypes binding of libb2attn.so (the C ABI in include/b2_decode_attn.h and
include/b2_block.h).

This module loads the in-tree shared library and nothing else: there is no
fallback.  If the library is missing or fails to load, every entry point
raises, so a GPU run can never silently take another path.
"""
from __future__ import annotations

import ctypes
import pathlib

LIB_PATH = pathlib.Path(__file__).resolve().parent / "libb2attn.so"

B2_OK = 0
B2_ERR_ARG = -1
B2_ERR_CUDA = -2
B2_ERR_NOSYM = -3

B2_DEV_BAD_BLOCK = 1
B2_DEV_BAD_LENGTH = 2
B2_DEV_BAD_POSITION = 4
B2_DEV_TIMEOUT = 8

B2_NORM_QK = 1
B2_ROPE_QK = 2
B2_STORE_KV = 4
B2_TEST_STALL = 0x100         # b2_decode_step test mode: one warp's wait runs out

B2_NOALLOC_MAX_PARTS = 1024   # batch * num_splits limit of b2_decode_attn_noalloc
B2_XCHG_MAX_WORLD = 8         # ranks of b2_exchange_merge

B2_GEMM_PLAIN = 0             # b2_gemm epilogues
B2_GEMM_SWIGLU = 1

DEV_ERR_NAMES = {
    B2_DEV_BAD_BLOCK: "block table entry outside the pool",
    B2_DEV_BAD_LENGTH: "length or position outside the block table",
    B2_DEV_BAD_POSITION: "RoPE position outside the cos/sin table",
    B2_DEV_TIMEOUT: "a bounded device wait ran out",
}

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float

# name -> (restype, argtypes); the order mirrors the header.
SIGNATURES = {
    "b2_version": (ctypes.c_int, []),
    "b2_last_error": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int]),
    "b2_set_wait_limits": (ctypes.c_int, [_i64, _i64]),
    "b2_get_wait_limits": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]),
    "b2_append_rope": (ctypes.c_int, [
        _p, _i64,            # qkv, row_stride
        _p, _p, _f32,        # gamma_q, gamma_k, eps
        _p, _p, _i32,        # rope_cos, rope_sin, rope_rows
        _p,                  # past_lens
        _p, _i32,            # block_tables, max_blocks_per_seq
        _p, _p, _i32,        # k_pool, v_pool, num_blocks
        _p, _i32, _i32,      # q_out, batch, mode
        _p, _p,              # dev_err, stream
    ]),
    "b2_decode_attn": (ctypes.c_int, [
        _p, _p, _p, _i32,    # q, k_pool, v_pool, num_blocks
        _p, _i32,            # block_tables, max_blocks_per_seq
        _p, _i32,            # seq_lens, batch
        _i32, _i32, _f32,    # blocks_per_split, num_splits, scale
        _p, _p,              # part_ml, part_o
        _p, _p,              # dev_err, stream
    ]),
    "b2_decode_step_counters": (ctypes.c_int, [_i32]),
    "b2_decode_step": (ctypes.c_int, [
        _p, _i64,            # qkv, row_stride
        _p, _p, _f32,        # gamma_q, gamma_k, eps
        _p, _p, _i32,        # rope_cos, rope_sin, rope_rows
        _p, _p,              # past_lens, seq_lens
        _p, _i32,            # block_tables, max_blocks_per_seq
        _p, _p, _i32,        # k_pool, v_pool, num_blocks
        _i32, _i32, _f32,    # batch, blocks_per_split, scale
        _i32, _p, _p,        # mode, out, q_out
        _p, _p,              # state_ml, state_o
        _p, _p, _p,          # part_ml, part_o, counters
        _i32, _p, _p,        # max_ctas, dev_err, stream
    ]),
    "b2_decode_step_host": (ctypes.c_int, [
        _p, _p, _p,          # qkv_host, past_host, out_host
        _p, _p, _p,          # qkv_dev, past_dev, out_dev
        _p, _p, _f32,        # gamma_q, gamma_k, eps
        _p, _p, _i32,        # rope_cos, rope_sin, rope_rows
        _p, _i32,            # block_tables, max_blocks_per_seq
        _p, _p, _i32,        # k_pool, v_pool, num_blocks
        _i32, _i32, _f32,    # batch, blocks_per_split, scale
        _p, _p, _p, _p,      # part_ml, part_o, counters, dev_err
        _p,                  # stream
    ]),
    "b2_decode_step_host2": (ctypes.c_int, [
        _p, _p, _p,          # qkv_host, past_host, out_host
        _p, _p, _p, _i32,    # qkv_dev2, past_dev2, out_dev2, slot
        _p, _p, _f32,        # gamma_q, gamma_k, eps
        _p, _p, _i32,        # rope_cos, rope_sin, rope_rows
        _p, _i32,            # block_tables, max_blocks_per_seq
        _p, _p, _i32,        # k_pool, v_pool, num_blocks
        _i32, _i32, _f32,    # batch, blocks_per_split, scale
        _p, _p, _p, _p,      # part_ml, part_o, counters, dev_err
        _p,                  # stream
    ]),
    "b2_decode_step_host_join": (ctypes.c_int, [_p]),
    "b2_prefill_attn_split": (ctypes.c_int, [
        _p, _p, _p, _i32,    # q, k_pool, v_pool, num_blocks
        _p, _i32,            # block_tables, max_blocks_per_seq
        _p, _p, _i32, _i32,  # past_lens, chunk_lens, tokens, batch
        _f32, _i32,          # scale, blocks_per_split
        _p, _p, _p, _p, _p,  # part_ml, part_o, out, dev_err, stream
    ]),
    "b2_decode_step_tokens": (ctypes.c_int, [
        _p, ctypes.c_int64, _i32, _p,  # qkv, row_stride, tokens, chunk_lens
        _p, _p, _f32,        # gamma_q, gamma_k, eps
        _p, _p, _i32,        # rope_cos, rope_sin, rope_rows
        _p, _p, _i32,        # past_lens, block_tables, max_blocks_per_seq
        _p, _p, _i32,        # k_pool, v_pool, num_blocks
        _i32, _i32, _f32, _i32,  # batch, blocks_per_split, scale, mode
        _p, _p, _p, _p,      # out, q_out, part_ml, part_o
        _p, _i32, _p, _p,    # counters, max_ctas, dev_err, stream
    ]),
    "b2_decode_step_exchange": (ctypes.c_int, [
        _p, ctypes.c_int64,  # qkv, row_stride
        _p, _p, _f32,        # gamma_q, gamma_k, eps
        _p, _p, _i32,        # rope_cos, rope_sin, rope_rows
        _p, _p,              # past_lens, seq_lens
        _p, _i32,            # block_tables, max_blocks_per_seq
        _p, _p, _i32,        # k_pool, v_pool, num_blocks
        _i32, _i32, _f32, _i32,  # batch, blocks_per_split, scale, mode
        _p, _p,              # out, q_out
        _p, _p, _p, _i32,    # part_ml, part_o, counters, max_ctas
        _p, _i32, _i32,      # areas (host array of world pointers), world, rank
        _p, _p,              # dev_err, stream
    ]),
    "b2_exchange_bytes": (ctypes.c_int64, [_i32, _i32]),
    "b2_ipc_handle": (ctypes.c_int, [_p, _p, ctypes.POINTER(ctypes.c_int64)]),
    "b2_ipc_open": (ctypes.c_int, [_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p)]),
    "b2_ipc_close": (ctypes.c_int, [_p, ctypes.c_int64]),
    "b2_exchange_merge": (ctypes.c_int, [
        _p, _p, _i32,        # state_ml, state_o, batch
        _p, _i32, _i32,      # areas (host array of world pointers), world, rank
        _p, _p, _p,          # out, dev_err, stream
    ]),
    # include/b2_block.h
    "b2_add_rmsnorm": (ctypes.c_int, [_p, _p, _p, _f32, _p, _p, _i32, _i32, _p]),
    "b2_swiglu": (ctypes.c_int, [_p, _p, _i32, _i32, _p]),
    "b2_shortconv_step": (ctypes.c_int, [_p, _p, _p, _p, _i32, _i32, _p]),
    "b2_argmax_rows": (ctypes.c_int, [_p, _i32, _i32, _p, _p]),
    "b2_gemm": (ctypes.c_int, [
        _p, _i64, _p, _i64,  # a, lda, w, ldw
        _p, _i64,            # d, ldd
        _i32, _i32, _i32,    # m, n, k
        _i32, _i32, _i32,    # mode, tile_n, splits
        _p, _p,              # dev_err, stream
    ]),
    "b2_gemm_plan": (ctypes.c_int, [_i32, _i32, _i32, _i32, ctypes.POINTER(ctypes.c_int32),
                                    ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]),
    "b2_merge_states": (ctypes.c_int, [
        _p, _i32, _i32,      # states, num_parts, batch
        _p, _p, _p, _p,      # out, state_ml, state_o, stream
    ]),
    "b2_prefill_append": (ctypes.c_int, [
        _p, _i64,            # qkv, row_stride
        _p, _p, _f32,        # gamma_q, gamma_k, eps
        _p, _p, _i32,        # rope_cos, rope_sin, rope_rows
        _p, _p, _i32,        # past_lens, chunk_lens, tokens
        _p, _i32,            # block_tables, max_blocks_per_seq
        _p, _p, _i32,        # k_pool, v_pool, num_blocks
        _p, _i32, _i32,      # q_out, batch, mode
        _p, _p,              # dev_err, stream
    ]),
    "b2_prefill_attn": (ctypes.c_int, [
        _p, _p, _p, _i32,    # q, k_pool, v_pool, num_blocks
        _p, _i32,            # block_tables, max_blocks_per_seq
        _p, _p, _i32, _i32,  # past_lens, chunk_lens, tokens, batch
        _f32, _p, _p, _p,    # scale, out, dev_err, stream
    ]),
    "b2_decode_attn_noalloc": (ctypes.c_int, [
        _p, _p, _p, _i32,    # q, k_pool, v_pool, num_blocks
        _p, _i32,            # block_tables, max_blocks_per_seq
        _p, _i32,            # seq_lens, batch
        _i32, _f32,          # blocks_per_split, scale
        _p, _p, _p,          # out, dev_err, stream
    ]),
    "b2_combine": (ctypes.c_int, [
        _p, _p, _i32,        # part_ml, part_o, num_parts
        _p, _i32, _i32,      # seq_lens, blocks_per_split, batch
        _p, _p, _p,          # out, state_ml, state_o
        _p,                  # stream
    ]),
}

_LIB = None


class B2Error(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{message} (status {code})")
        self.code = code


def load() -> ctypes.CDLL:
    """Load libb2attn.so once and bind every exported entry point."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH.name} is not built; run __graft_entry__.build() "
            f"(or python {LIB_PATH.parent.name}/build.py)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().b2_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, call: str) -> None:
    if status != B2_OK:
        raise B2Error(status, f"{call}: {last_error()}")


def set_wait_limits(wait_ns: int = 0, poll_ns: int = 0) -> None:
    """Limits of the kernels' bounded waits for later launches (0: defaults,
    2 s for a wait on another warp, 5 s for the multi-GPU exchange's poll)."""
    check(load().b2_set_wait_limits(int(wait_ns), int(poll_ns)), "b2_set_wait_limits")


def get_wait_limits() -> tuple[int, int]:
    w, p = ctypes.c_int64(), ctypes.c_int64()
    check(load().b2_get_wait_limits(ctypes.byref(w), ctypes.byref(p)), "b2_get_wait_limits")
    return w.value, p.value


def decode_dev_err(word: int) -> list[str]:
    return [text for bit, text in DEV_ERR_NAMES.items() if word & bit]
