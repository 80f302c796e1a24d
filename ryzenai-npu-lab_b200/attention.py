"""Torch-facing wrappers over the C ABI, and the decode-attention runner.

PyTorch provides device memory and streams here; every byte of attention
math runs in libb2attn.so (see _lib.py).  Each wrapper checks dtypes, shapes,
devices and contiguity on the host (raising ValueError like the reference's
operators, e.g. experiments/lfm25_attention_context_cache_kernel.py:25-26) and
raises B2Error when the library refuses a call.  Device-side faults (a bad
block id, a length beyond the block table) are collected in a device word
that `PagedDecodeAttention.check()` reads and turns into RuntimeError, like
the reference's failed-run check (experiments/npu_direct.py:110-114).
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .paged_cache import BLOCK, PagedKVCache
from .rope import rope_table

HQ, HKV, D = 16, 8, 64
QKV_WIDTH = (HQ + 2 * HKV) * D
SCALE = D ** -0.5
EPS = 1.0e-5
B200_SMS = 148


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device, stream: torch.cuda.Stream | None):
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return ctypes.c_void_p(s.cuda_stream)


def _need(t: torch.Tensor, name: str, dtype: torch.dtype, device: torch.device, shape=None):
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{name} must be a tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if t.device != device:
        raise ValueError(f"{name} must be on {device}, got {t.device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")


def _need_rope(cos, sin, device: torch.device) -> int:
    """cos/sin tables bf16 [positions, 64] (one row per RoPE position); returns positions."""
    _need(cos, "cos", torch.bfloat16, device)
    _need(sin, "sin", torch.bfloat16, device, tuple(cos.shape))
    if cos.dim() != 2 or cos.shape[1] != D or cos.shape[0] == 0:
        raise ValueError(f"cos/sin must be [positions >= 1, {D}], got {tuple(cos.shape)}")
    return cos.shape[0]


def append_rope(qkv: torch.Tensor, past_lens: torch.Tensor, *, q_out: torch.Tensor | None,
                dev_err: torch.Tensor, mode: int = _lib.B2_NORM_QK | _lib.B2_ROPE_QK | _lib.B2_STORE_KV,
                gamma_q: torch.Tensor | None = None, gamma_k: torch.Tensor | None = None,
                cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                k_pool: torch.Tensor | None = None, v_pool: torch.Tensor | None = None,
                block_tables: torch.Tensor | None = None, eps: float = EPS,
                stream: torch.cuda.Stream | None = None) -> None:
    """q/k RMSNorm + RoPE at position past_lens[b] + write of k, v into slot
    past_lens[b] of the pool (b2_append_rope).  qkv: bf16 [B, W >= 2048]."""
    dev = qkv.device
    if qkv.dim() != 2 or qkv.shape[1] < QKV_WIDTH:
        raise ValueError(f"qkv must be [batch, >= {QKV_WIDTH}], got {tuple(qkv.shape)}")
    _need(qkv, "qkv", torch.bfloat16, dev)
    b = qkv.shape[0]
    _need(past_lens, "past_lens", torch.int32, dev, (b,))
    _need(dev_err, "dev_err", torch.int32, dev)
    if q_out is not None:
        _need(q_out, "q_out", torch.bfloat16, dev, (b, HQ, D))
    rope_rows = 0
    if mode & _lib.B2_NORM_QK:
        _need(gamma_q, "gamma_q", torch.bfloat16, dev, (D,))
        _need(gamma_k, "gamma_k", torch.bfloat16, dev, (D,))
    if mode & _lib.B2_ROPE_QK:
        rope_rows = _need_rope(cos, sin, dev)
    max_blocks = num_blocks = 0
    if mode & _lib.B2_STORE_KV:
        _need(k_pool, "k_pool", torch.bfloat16, dev)
        _need(v_pool, "v_pool", torch.bfloat16, dev, tuple(k_pool.shape))
        if k_pool.dim() != 4 or tuple(k_pool.shape[1:]) != (HKV, BLOCK, D):
            raise ValueError("pools must be [num_blocks, 8, 64, 64]")
        _need(block_tables, "block_tables", torch.int32, dev)
        if block_tables.dim() != 2 or block_tables.shape[0] != b:
            raise ValueError("block_tables must be [batch, max_blocks_per_seq]")
        max_blocks, num_blocks = block_tables.shape[1], k_pool.shape[0]
    rc = _lib.load().b2_append_rope(
        _ptr(qkv), qkv.stride(0), _ptr(gamma_q), _ptr(gamma_k), ctypes.c_float(eps),
        _ptr(cos), _ptr(sin), rope_rows, _ptr(past_lens), _ptr(block_tables), max_blocks,
        _ptr(k_pool), _ptr(v_pool), num_blocks, _ptr(q_out), b, mode, _ptr(dev_err),
        _stream(dev, stream))
    _lib.check(rc, "b2_append_rope")


def num_splits_for(max_blocks: int, blocks_per_split: int) -> int:
    return max(1, (max_blocks + blocks_per_split - 1) // blocks_per_split)


def choose_blocks_per_split(batch: int, work_blocks: int, sms: int = B200_SMS, fused: bool = False,
                            max_blocks_per_seq: int | None = None) -> int:
    """Blocks per work item.  work_blocks: total 64-token blocks over the
    batch (one head).  Three-kernel path: about 8 CTAs of real work per SM
    (3 are resident at a time; the rest balance the tail).  Fused persistent
    kernel: about 6 items per resident CTA (items stream back to back, so they
    can be smaller; the end-of-launch tail is one item), at least 6 blocks.
    Measured on the C3 workload: the fused kernel is within 1 % of its best for
    8-16 blocks; on its shards (8 / 16 / 32 sequences) the best are 6 / 6 / 8
    blocks.  With many sequences of at most 32 blocks, one split per sequence.
    The split grows to ceil(longest / 16) blocks when that still leaves about
    3 items per resident CTA, so that a sequence has at most 16 splits and the
    kernel's merger warp merges them without a combine launch.
    With a few sequences (a long context split over the CTAs) the items are
    all alike: about two per SM in one wave, every CTA streaming the same
    number of blocks (up to 64), finish together; measured on one 131 072-token
    sequence: 46.9 us at 296 items against 51.4 us at 432 and 52 us at 2 056."""
    if fused:
        # the longest sequence (the block-table width) when known, else the mean
        per_seq_max = max_blocks_per_seq or math.ceil(work_blocks / max(1, batch))
        if batch * HKV >= 2 * sms * 3 and per_seq_max <= 32:
            # many short sequences: one split each (no cross-CTA merge; the
            # item's own epilogue writes the context)
            return int(max(1, per_seq_max))
        if batch <= 4:
            per_seq = math.ceil(work_blocks / max(1, batch))
            splits = max(1, (sms * 2) // (max(1, batch) * HKV))
            return int(max(1, min(64, math.ceil(per_seq / splits))))
        bps = int(min(32, max(6, math.ceil(work_blocks * HKV / (sms * 3 * 6)))))
        # at most 16 splits per sequence (merged by the kernel's merger warp, no
        # combine launch) when that still leaves ~3 items per resident CTA
        merge_bps = math.ceil(per_seq_max / 16)
        items = HKV * (work_blocks / merge_bps + batch)
        if bps < merge_bps <= 64 and items >= 3 * (3 * sms):
            bps = int(merge_bps)
        return bps
    target = 8 * sms
    return int(min(64, max(2, math.ceil(work_blocks * HKV / target))))


def decode_attn(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                block_tables: torch.Tensor, seq_lens: torch.Tensor, *, blocks_per_split: int,
                part_ml: torch.Tensor, part_o: torch.Tensor, dev_err: torch.Tensor,
                scale: float = SCALE, stream: torch.cuda.Stream | None = None) -> int:
    """Split-KV decode (b2_decode_attn) into partial states; returns num_splits."""
    dev = q.device
    b = q.shape[0]
    _need(q, "q", torch.bfloat16, dev, (b, HQ, D))
    _need(k_pool, "k_pool", torch.bfloat16, dev)
    _need(v_pool, "v_pool", torch.bfloat16, dev, tuple(k_pool.shape))
    if k_pool.dim() != 4 or tuple(k_pool.shape[1:]) != (HKV, BLOCK, D):
        raise ValueError("pools must be [num_blocks, 8, 64, 64]")
    _need(block_tables, "block_tables", torch.int32, dev)
    if block_tables.dim() != 2 or block_tables.shape[0] != b:
        raise ValueError("block_tables must be [batch, max_blocks_per_seq]")
    _need(seq_lens, "seq_lens", torch.int32, dev, (b,))
    max_blocks = block_tables.shape[1]
    splits = num_splits_for(max_blocks, blocks_per_split)
    _need(part_ml, "part_ml", torch.float32, dev)
    _need(part_o, "part_o", torch.float32, dev)
    if part_ml.numel() < b * splits * HQ * 2 or part_o.numel() < b * splits * HQ * D:
        raise ValueError(f"partial-state buffers too small for {b} x {splits} splits")
    rc = _lib.load().b2_decode_attn(
        _ptr(q), _ptr(k_pool), _ptr(v_pool), k_pool.shape[0], _ptr(block_tables), max_blocks,
        _ptr(seq_lens), b, blocks_per_split, splits, ctypes.c_float(scale), _ptr(part_ml),
        _ptr(part_o), _ptr(dev_err), _stream(dev, stream))
    _lib.check(rc, "b2_decode_attn")
    return splits


def combine(part_ml: torch.Tensor, part_o: torch.Tensor, num_parts: int, batch: int, *,
            seq_lens: torch.Tensor | None = None, blocks_per_split: int = 1,
            out: torch.Tensor | None = None, state_ml: torch.Tensor | None = None,
            state_o: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> None:
    """Log-sum-exp merge (b2_combine) into bf16 out [B, 16, 64] and/or a merged
    fp32 state (state_ml [B, 16, 2], state_o [B, 16, 64])."""
    dev = part_ml.device
    _need(part_ml, "part_ml", torch.float32, dev)
    _need(part_o, "part_o", torch.float32, dev)
    if part_ml.numel() < batch * num_parts * HQ * 2 or part_o.numel() < batch * num_parts * HQ * D:
        raise ValueError("partial-state buffers smaller than batch x num_parts")
    if seq_lens is not None:
        _need(seq_lens, "seq_lens", torch.int32, dev, (batch,))
    if out is not None:
        _need(out, "out", torch.bfloat16, dev)
        if out.numel() != batch * HQ * D:
            raise ValueError("out must hold batch x 16 x 64 elements")
    if state_o is not None:
        _need(state_ml, "state_ml", torch.float32, dev, (batch, HQ, 2))
        _need(state_o, "state_o", torch.float32, dev, (batch, HQ, D))
    rc = _lib.load().b2_combine(
        _ptr(part_ml), _ptr(part_o), num_parts, _ptr(seq_lens), blocks_per_split, batch,
        _ptr(out), _ptr(state_ml), _ptr(state_o), _stream(dev, stream))
    _lib.check(rc, "b2_combine")


def decode_step(qkv: torch.Tensor, past_lens: torch.Tensor, *, k_pool: torch.Tensor, v_pool: torch.Tensor,
                block_tables: torch.Tensor, blocks_per_split: int, out: torch.Tensor | None,
                part_ml: torch.Tensor, part_o: torch.Tensor, counters: torch.Tensor, dev_err: torch.Tensor,
                gamma_q: torch.Tensor | None = None, gamma_k: torch.Tensor | None = None,
                cos: torch.Tensor | None = None, sin: torch.Tensor | None = None, q_out: torch.Tensor | None = None,
                seq_lens: torch.Tensor | None = None, state_ml: torch.Tensor | None = None,
                state_o: torch.Tensor | None = None,
                mode: int = _lib.B2_NORM_QK | _lib.B2_ROPE_QK | _lib.B2_STORE_KV, eps: float = EPS,
                scale: float = SCALE, max_ctas: int = 0, stream: torch.cuda.Stream | None = None,
                exchange=None) -> int:
    """Fused decode step in one persistent launch (b2_decode_step): norm + RoPE,
    append at past_lens[b], attention over past_lens[b] + 1 tokens (or
    seq_lens[b]), merge into `out` or into fp32 states (state_ml, state_o).
    With exchange = (areas, world, rank) (b2_decode_step_exchange) the merged
    states are exchanged with the other ranks over peer memory and `out`
    receives the world's context.  `counters` (int32[2 + 8 * batch]) must be
    zero on the first call; the kernel leaves it zero.  Returns num_splits."""
    dev = qkv.device
    if qkv.dim() != 2 or qkv.shape[1] < QKV_WIDTH:
        raise ValueError(f"qkv must be [batch, >= {QKV_WIDTH}], got {tuple(qkv.shape)}")
    _need(qkv, "qkv", torch.bfloat16, dev)
    b = qkv.shape[0]
    _need(past_lens, "past_lens", torch.int32, dev, (b,))
    _need(k_pool, "k_pool", torch.bfloat16, dev)
    _need(v_pool, "v_pool", torch.bfloat16, dev, tuple(k_pool.shape))
    if k_pool.dim() != 4 or tuple(k_pool.shape[1:]) != (HKV, BLOCK, D):
        raise ValueError("pools must be [num_blocks, 8, 64, 64]")
    _need(block_tables, "block_tables", torch.int32, dev)
    if block_tables.dim() != 2 or block_tables.shape[0] != b:
        raise ValueError("block_tables must be [batch, max_blocks_per_seq]")
    if out is not None:
        _need(out, "out", torch.bfloat16, dev)
        if out.numel() != b * HQ * D:
            raise ValueError("out must hold batch x 16 x 64 elements")
    if exchange is not None:
        if out is None or state_o is not None or state_ml is not None:
            raise ValueError("a decode step with an exchange writes out and no state")
    elif state_o is not None or out is None:
        _need(state_ml, "state_ml", torch.float32, dev, (b, HQ, 2))
        _need(state_o, "state_o", torch.float32, dev, (b, HQ, D))
    if seq_lens is not None:
        _need(seq_lens, "seq_lens", torch.int32, dev, (b,))
    if q_out is not None:
        _need(q_out, "q_out", torch.bfloat16, dev, (b, HQ, D))
    _need(counters, "counters", torch.int32, dev)
    if counters.numel() < 2 + HKV * b:
        raise ValueError("counters must hold 2 + 8 * batch int32")
    _need(dev_err, "dev_err", torch.int32, dev)
    rope_rows = 0
    if mode & _lib.B2_NORM_QK:
        _need(gamma_q, "gamma_q", torch.bfloat16, dev, (D,))
        _need(gamma_k, "gamma_k", torch.bfloat16, dev, (D,))
    if mode & _lib.B2_ROPE_QK:
        rope_rows = _need_rope(cos, sin, dev)
    max_blocks = block_tables.shape[1]
    splits = num_splits_for(max_blocks, blocks_per_split)
    _need(part_ml, "part_ml", torch.float32, dev)
    _need(part_o, "part_o", torch.float32, dev)
    if part_ml.numel() < b * splits * HQ * 2 or part_o.numel() < b * splits * HQ * D:
        raise ValueError(f"partial-state buffers too small for {b} x {splits} splits")
    common = (_ptr(qkv), qkv.stride(0), _ptr(gamma_q), _ptr(gamma_k), ctypes.c_float(eps), _ptr(cos), _ptr(sin),
              rope_rows, _ptr(past_lens), _ptr(seq_lens), _ptr(block_tables), max_blocks, _ptr(k_pool),
              _ptr(v_pool), k_pool.shape[0], b, blocks_per_split, ctypes.c_float(scale), mode, _ptr(out),
              _ptr(q_out))
    if exchange is not None:
        areas, world, rank = exchange
        rc = _lib.load().b2_decode_step_exchange(*common, _ptr(part_ml), _ptr(part_o), _ptr(counters), max_ctas,
                                                 areas, world, rank, _ptr(dev_err), _stream(dev, stream))
        _lib.check(rc, "b2_decode_step_exchange")
        return splits
    rc = _lib.load().b2_decode_step(*common, _ptr(state_ml), _ptr(state_o), _ptr(part_ml), _ptr(part_o),
                                    _ptr(counters), max_ctas, _ptr(dev_err), _stream(dev, stream))
    _lib.check(rc, "b2_decode_step")
    return splits


MAX_STEP_TOKENS = 4   # new tokens per sequence of b2_decode_step_tokens
MAX_MERGED_SPLITS = 16


def step_tokens_blocks_per_split(batch: int, max_blocks: int, sms: int = B200_SMS) -> int:
    """Split size for b2_decode_step_tokens: the decode step's heuristic, but
    at most 16 splits per sequence (the kernel merges them itself)."""
    bps = choose_blocks_per_split(batch, batch * max_blocks, sms, fused=True, max_blocks_per_seq=max_blocks)
    return int(max(bps, math.ceil(max_blocks / MAX_MERGED_SPLITS)))


def decode_step_tokens(qkv: torch.Tensor, past_lens: torch.Tensor, *, k_pool: torch.Tensor, v_pool: torch.Tensor,
                       block_tables: torch.Tensor, out: torch.Tensor, counters: torch.Tensor,
                       dev_err: torch.Tensor, blocks_per_split: int | None = None,
                       part_ml: torch.Tensor | None = None, part_o: torch.Tensor | None = None,
                       gamma_q: torch.Tensor | None = None, gamma_k: torch.Tensor | None = None,
                       cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                       q_out: torch.Tensor | None = None, chunk_lens: torch.Tensor | None = None,
                       mode: int = _lib.B2_NORM_QK | _lib.B2_ROPE_QK | _lib.B2_STORE_KV, eps: float = EPS,
                       scale: float = SCALE, max_ctas: int = 0, stream: torch.cuda.Stream | None = None) -> int:
    """The fused decode step for T = 1..4 new tokens per sequence
    (b2_decode_step_tokens): qkv bf16 [B, T, >= 2048] raw projections of the
    tokens at positions past_lens[b] + t (chunk_lens[b] of them valid, all
    when None); appends their k/v, writes the contexts out [B, T, 16, 64]
    (token t attends the cache and the new tokens up to itself).  Returns the
    number of splits."""
    dev = qkv.device
    if qkv.dim() != 3 or qkv.shape[2] < QKV_WIDTH:
        raise ValueError(f"qkv must be [batch, tokens, >= {QKV_WIDTH}], got {tuple(qkv.shape)}")
    b, t = qkv.shape[0], qkv.shape[1]
    if not 1 <= t <= MAX_STEP_TOKENS:
        raise ValueError(f"tokens must be in [1, {MAX_STEP_TOKENS}], got {t}")
    if qkv.dtype != torch.bfloat16 or qkv.device != dev or qkv.stride(2) != 1 or qkv.stride(0) != t * qkv.stride(1):
        raise ValueError("qkv must be bf16 with rows b * tokens + t at a common stride")
    _need(past_lens, "past_lens", torch.int32, dev, (b,))
    if chunk_lens is not None:
        _need(chunk_lens, "chunk_lens", torch.int32, dev, (b,))
    _need(k_pool, "k_pool", torch.bfloat16, dev)
    _need(v_pool, "v_pool", torch.bfloat16, dev, tuple(k_pool.shape))
    if k_pool.dim() != 4 or tuple(k_pool.shape[1:]) != (HKV, BLOCK, D):
        raise ValueError("pools must be [num_blocks, 8, 64, 64]")
    _need(block_tables, "block_tables", torch.int32, dev)
    if block_tables.dim() != 2 or block_tables.shape[0] != b:
        raise ValueError("block_tables must be [batch, max_blocks_per_seq]")
    _need(out, "out", torch.bfloat16, dev, (b, t, HQ, D))
    if q_out is not None:
        _need(q_out, "q_out", torch.bfloat16, dev, (b, t, HQ, D))
    _need(counters, "counters", torch.int32, dev)
    if counters.numel() < 2 + HKV * b:
        raise ValueError("counters must hold 2 + 8 * batch int32")
    _need(dev_err, "dev_err", torch.int32, dev)
    rope_rows = 0
    if mode & _lib.B2_NORM_QK:
        _need(gamma_q, "gamma_q", torch.bfloat16, dev, (D,))
        _need(gamma_k, "gamma_k", torch.bfloat16, dev, (D,))
    if mode & _lib.B2_ROPE_QK:
        rope_rows = _need_rope(cos, sin, dev)
    max_blocks = block_tables.shape[1]
    bps = blocks_per_split or step_tokens_blocks_per_split(b, max_blocks)
    splits = num_splits_for(max_blocks, bps)
    if part_ml is None:
        part_ml = torch.empty(b, t, splits, HQ, 2, dtype=torch.float32, device=dev)
    if part_o is None:
        part_o = torch.empty(b, t, splits, HQ, D, dtype=torch.float32, device=dev)
    _need(part_ml, "part_ml", torch.float32, dev)
    _need(part_o, "part_o", torch.float32, dev)
    if part_ml.numel() < b * t * splits * HQ * 2 or part_o.numel() < b * t * splits * HQ * D:
        raise ValueError(f"partial-state buffers too small for {b} x {t} x {splits} splits")
    rc = _lib.load().b2_decode_step_tokens(
        _ptr(qkv), qkv.stride(1), t, _ptr(chunk_lens), _ptr(gamma_q), _ptr(gamma_k), ctypes.c_float(eps), _ptr(cos),
        _ptr(sin), rope_rows, _ptr(past_lens), _ptr(block_tables), max_blocks, _ptr(k_pool), _ptr(v_pool),
        k_pool.shape[0], b, bps, ctypes.c_float(scale), mode, _ptr(out), _ptr(q_out), _ptr(part_ml), _ptr(part_o),
        _ptr(counters), max_ctas, _ptr(dev_err), _stream(dev, stream))
    _lib.check(rc, "b2_decode_step_tokens")
    return splits


def merge_states(states: torch.Tensor, num_parts: int, batch: int, *, out: torch.Tensor | None = None,
                 state_ml: torch.Tensor | None = None, state_o: torch.Tensor | None = None,
                 stream: torch.cuda.Stream | None = None) -> None:
    """Merge states gathered from num_parts GPUs (b2_merge_states): `states`
    is fp32 [num_parts, batch * 16 * 66], each part [ml batch*16*2 | o batch*16*64]."""
    dev = states.device
    _need(states, "states", torch.float32, dev)
    if states.numel() != num_parts * batch * HQ * (2 + D):
        raise ValueError("states must hold num_parts x batch x 16 x 66 floats")
    if out is not None:
        _need(out, "out", torch.bfloat16, dev)
        if out.numel() != batch * HQ * D:
            raise ValueError("out must hold batch x 16 x 64 elements")
    if state_o is not None:
        _need(state_ml, "state_ml", torch.float32, dev, (batch, HQ, 2))
        _need(state_o, "state_o", torch.float32, dev, (batch, HQ, D))
    rc = _lib.load().b2_merge_states(_ptr(states), num_parts, batch, _ptr(out), _ptr(state_ml), _ptr(state_o),
                                     _stream(dev, stream))
    _lib.check(rc, "b2_merge_states")


def prefill(qkv: torch.Tensor, past_lens: torch.Tensor, *, k_pool: torch.Tensor, v_pool: torch.Tensor,
            block_tables: torch.Tensor, gamma_q: torch.Tensor | None, gamma_k: torch.Tensor | None,
            cos: torch.Tensor | None, sin: torch.Tensor | None, dev_err: torch.Tensor,
            chunk_lens: torch.Tensor | None = None, out: torch.Tensor | None = None,
            q_out: torch.Tensor | None = None, eps: float = EPS, scale: float = SCALE,
            mode: int = _lib.B2_NORM_QK | _lib.B2_ROPE_QK | _lib.B2_STORE_KV,
            blocks_per_split: int | None = None, stream: torch.cuda.Stream | None = None,
            kernel: str = "auto") -> torch.Tensor:
    """Batched-prompt attention (b2_prefill_append + b2_prefill_attn): qkv bf16
    [B, T, >= 2048] raw projections of T new tokens per sequence at positions
    past_lens[b] + t (chunk_lens[b] <= T valid).  Appends their k/v and returns
    the context [B, T, 16, 64].  `mode` selects the q/k norm and RoPE steps
    (B2_STORE_KV alone for projections that are already normalised and rotated;
    gamma/cos/sin are then unused).  blocks_per_split > 0 splits every tile's
    keys over more CTAs (b2_prefill_attn_split; None = the heuristic
    prefill_blocks_per_split, 0 = no split).  kernel: "tcgen05" (the above),
    "step" (the fused decode step for up to 4 new tokens,
    b2_decode_step_tokens: 1.3-1.5x faster there; blocks_per_split is then its
    split size) or "auto" (the step for T <= 4 without chunk_lens when a
    sequence's keys fit 16 splits, else tcgen05)."""
    dev = qkv.device
    if qkv.dim() != 3 or qkv.shape[2] < QKV_WIDTH:
        raise ValueError(f"qkv must be [batch, tokens, >= {QKV_WIDTH}], got {tuple(qkv.shape)}")
    _need(qkv, "qkv", torch.bfloat16, dev)
    b, t = qkv.shape[0], qkv.shape[1]
    _need(past_lens, "past_lens", torch.int32, dev, (b,))
    if chunk_lens is not None:
        _need(chunk_lens, "chunk_lens", torch.int32, dev, (b,))
    _need(k_pool, "k_pool", torch.bfloat16, dev)
    _need(v_pool, "v_pool", torch.bfloat16, dev, tuple(k_pool.shape))
    if k_pool.dim() != 4 or tuple(k_pool.shape[1:]) != (HKV, BLOCK, D):
        raise ValueError("pools must be [num_blocks, 8, 64, 64]")
    _need(block_tables, "block_tables", torch.int32, dev)
    if block_tables.dim() != 2 or block_tables.shape[0] != b:
        raise ValueError("block_tables must be [batch, max_blocks_per_seq]")
    rope_rows = 0
    if mode & _lib.B2_NORM_QK:
        _need(gamma_q, "gamma_q", torch.bfloat16, dev, (D,))
        _need(gamma_k, "gamma_k", torch.bfloat16, dev, (D,))
    if mode & _lib.B2_ROPE_QK:
        rope_rows = _need_rope(cos, sin, dev)
    _need(dev_err, "dev_err", torch.int32, dev)
    if q_out is None:
        q_out = torch.empty(b, t, HQ, D, dtype=torch.bfloat16, device=dev)
    _need(q_out, "q_out", torch.bfloat16, dev, (b, t, HQ, D))
    if out is None:
        out = torch.empty(b, t, HQ, D, dtype=torch.bfloat16, device=dev)
    _need(out, "out", torch.bfloat16, dev, (b, t, HQ, D))
    if kernel not in ("auto", "step", "tcgen05"):
        raise ValueError("kernel must be auto, step or tcgen05")
    if kernel == "step" or (kernel == "auto" and t <= MAX_STEP_TOKENS and chunk_lens is None and
                            math.ceil(block_tables.shape[1] / MAX_MERGED_SPLITS) <= 64):
        counters = torch.zeros(2 + HKV * b, dtype=torch.int32, device=dev)
        decode_step_tokens(qkv, past_lens, k_pool=k_pool, v_pool=v_pool, block_tables=block_tables, out=out,
                           counters=counters, dev_err=dev_err, blocks_per_split=blocks_per_split or None,
                           gamma_q=gamma_q, gamma_k=gamma_k, cos=cos, sin=sin, q_out=q_out, chunk_lens=chunk_lens,
                           mode=mode, eps=eps, scale=scale, stream=stream)
        return out
    lib = _lib.load()
    st = _stream(dev, stream)
    rc = lib.b2_prefill_append(_ptr(qkv), qkv.stride(1), _ptr(gamma_q), _ptr(gamma_k), ctypes.c_float(eps),
                               _ptr(cos), _ptr(sin), rope_rows, _ptr(past_lens), _ptr(chunk_lens), t,
                               _ptr(block_tables), block_tables.shape[1], _ptr(k_pool), _ptr(v_pool),
                               k_pool.shape[0], _ptr(q_out), b, mode, _ptr(dev_err), st)
    _lib.check(rc, "b2_prefill_append")
    if blocks_per_split is None:
        blocks_per_split = prefill_blocks_per_split(b, t, block_tables.shape[1])
    if blocks_per_split > 0:
        nsplit = num_splits_for(block_tables.shape[1], blocks_per_split)
        part_ml = torch.empty(nsplit, b, t, HQ, 2, dtype=torch.float32, device=dev)
        part_o = torch.empty(nsplit, b, t, HQ, D, dtype=torch.float32, device=dev)
        rc = lib.b2_prefill_attn_split(_ptr(q_out), _ptr(k_pool), _ptr(v_pool), k_pool.shape[0],
                                       _ptr(block_tables), block_tables.shape[1], _ptr(past_lens),
                                       _ptr(chunk_lens), t, b, ctypes.c_float(scale), blocks_per_split,
                                       _ptr(part_ml), _ptr(part_o), _ptr(out), _ptr(dev_err), st)
        _lib.check(rc, "b2_prefill_attn_split")
        return out
    rc = lib.b2_prefill_attn(_ptr(q_out), _ptr(k_pool), _ptr(v_pool), k_pool.shape[0], _ptr(block_tables),
                             block_tables.shape[1], _ptr(past_lens), _ptr(chunk_lens), t, b,
                             ctypes.c_float(scale), _ptr(out), _ptr(dev_err), st)
    _lib.check(rc, "b2_prefill_attn")
    return out


def prefill_blocks_per_split(batch: int, tokens: int, max_blocks: int, sms: int = B200_SMS) -> int:
    """Key split for b2_prefill_attn_split, 0 for none.  Only when the tiles
    alone give fewer CTAs than SMs (a few long sequences): then the keys are
    split so that about two CTAs per SM share the work, in ranges of at least
    16 blocks.  With a full GPU the split only adds partial states and a merge
    (measured on 64 sequences with 4-32 new tokens: 15-40 % slower)."""
    if batch <= 0 or tokens <= 0:
        return 0
    ctas = batch * HKV * math.ceil(tokens / 64)
    if ctas >= sms:
        return 0
    nsplit = min(math.ceil(2 * sms / ctas), math.ceil(max_blocks / 16))
    if nsplit <= 1 or batch * nsplit > 65535:
        return 0
    return int(math.ceil(max_blocks / nsplit))


class PagedDecodeAttention:
    """Decode attention of one new token per sequence over a PagedKVCache.

    step(layer, qkv, past_lens, seq_lens) runs, on the current stream, either
    the fused persistent kernel (b2_decode_step, the default) or the three
    separate kernels (fused=False):
      b2_append_rope  (q/k norm + RoPE, k/v into slot past_lens[b])
      b2_decode_attn  (split-KV flash-decode over seq_lens[b] tokens)
      b2_combine      (partial states -> bf16 context [B, 16, 64])
    seq_lens must equal past_lens + 1 (the new token is attended; the fused
    kernel derives it from past_lens).  All buffers are allocated here once;
    step() allocates nothing, so it can be captured in a CUDA graph.
    """

    def __init__(self, cache: PagedKVCache, gamma_q: torch.Tensor, gamma_k: torch.Tensor,
                 max_batch: int, rope_positions: int, *, eps: float = EPS,
                 blocks_per_split: int | None = None, work_blocks: int | None = None,
                 fused: bool = True, max_ctas: int = 0):
        self.cache = cache
        dev = cache.device
        self.device = dev
        self.eps = eps
        self.gamma_q = gamma_q.to(dev, torch.bfloat16).contiguous()
        self.gamma_k = gamma_k.to(dev, torch.bfloat16).contiguous()
        self.cos, self.sin = rope_table(rope_positions, device=dev)
        if blocks_per_split is None:
            wb = work_blocks if work_blocks is not None else max_batch * cache.max_blocks
            blocks_per_split = choose_blocks_per_split(max_batch, wb, fused=fused,
                                                       max_blocks_per_seq=cache.max_blocks)
        if fused and blocks_per_split > 64:
            raise ValueError("the fused kernel takes at most 64 blocks per split")
        self.blocks_per_split = blocks_per_split
        self.fused = fused
        self.max_ctas = max_ctas
        self.num_splits = num_splits_for(cache.max_blocks, blocks_per_split)
        self.max_batch = max_batch
        self.q = torch.empty(max_batch, HQ, D, dtype=torch.bfloat16, device=dev)
        self.part_ml = torch.empty(max_batch, self.num_splits, HQ, 2, dtype=torch.float32, device=dev)
        self.part_o = torch.empty(max_batch, self.num_splits, HQ, D, dtype=torch.float32, device=dev)
        self.out = torch.empty(max_batch, HQ, D, dtype=torch.bfloat16, device=dev)
        self.dev_err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.counters = torch.zeros(2 + HKV * max_batch, dtype=torch.int32, device=dev)

    def step(self, layer: int, qkv: torch.Tensor, past_lens: torch.Tensor, seq_lens: torch.Tensor,
             block_tables: torch.Tensor, out: torch.Tensor | None = None,
             stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        b = qkv.shape[0]
        if b > self.max_batch:
            raise ValueError(f"batch {b} > max_batch {self.max_batch}")
        kp, vp = self.cache.pool(layer)
        q = self.q[:b]
        if self.fused:
            o = self.out[:b] if out is None else out
            decode_step(qkv, past_lens, k_pool=kp, v_pool=vp, block_tables=block_tables,
                        blocks_per_split=self.blocks_per_split, out=o, part_ml=self.part_ml, part_o=self.part_o,
                        counters=self.counters, dev_err=self.dev_err, gamma_q=self.gamma_q, gamma_k=self.gamma_k,
                        cos=self.cos, sin=self.sin, q_out=q, eps=self.eps, max_ctas=self.max_ctas, stream=stream)
            return o
        append_rope(qkv, past_lens, q_out=q, dev_err=self.dev_err, gamma_q=self.gamma_q,
                    gamma_k=self.gamma_k, cos=self.cos, sin=self.sin, k_pool=kp, v_pool=vp,
                    block_tables=block_tables, eps=self.eps, stream=stream)
        splits = decode_attn(q, kp, vp, block_tables, seq_lens, blocks_per_split=self.blocks_per_split,
                             part_ml=self.part_ml, part_o=self.part_o, dev_err=self.dev_err,
                             stream=stream)
        o = self.out[:b] if out is None else out
        combine(self.part_ml, self.part_o, splits, b, seq_lens=seq_lens,
                blocks_per_split=self.blocks_per_split, out=o, stream=stream)
        return o

    # ---------------------------------------------------------------- host-fed steps

    def open_host_pipeline(self, layer: int, block_tables: torch.Tensor, batch: int | None = None,
                           double_buffered: bool = True) -> None:
        """Prepare step_host(): device staging buffers and the C-ABI arguments,
        validated once here, not per step.  double_buffered selects
        b2_decode_step_host2 (two staging slots; copies on library-owned
        streams overlap the neighbouring kernels) over b2_decode_step_host
        (one slot; copies and kernel in the caller's stream order)."""
        if not self.fused:
            raise ValueError("the host-fed step runs the fused kernel")
        b = self.max_batch if batch is None else batch
        dev = self.device
        _need(block_tables, "block_tables", torch.int32, dev)
        if block_tables.dim() != 2 or block_tables.shape[0] != b:
            raise ValueError("block_tables must be [batch, max_blocks_per_seq]")
        splits = num_splits_for(block_tables.shape[1], self.blocks_per_split)
        if self.part_ml.numel() < b * splits * HQ * 2:
            raise ValueError("partial-state buffers too small")
        kp, vp = self.cache.pool(layer)
        slots = 2 if double_buffered else 1
        hp = {"b": b, "tables": block_tables, "slot": 0, "double": double_buffered, "pinned": set(),
              "qkv": torch.empty(slots, b, QKV_WIDTH, dtype=torch.bfloat16, device=dev),
              "past": torch.empty(slots, b, dtype=torch.int32, device=dev),
              "out": torch.empty(slots, b, HQ, D, dtype=torch.bfloat16, device=dev)}
        lib = _lib.load()
        hp["call"] = lib.b2_decode_step_host2 if double_buffered else lib.b2_decode_step_host
        hp["join"] = lib.b2_decode_step_host_join
        hp["bufs"] = (_ptr(hp["qkv"]), _ptr(hp["past"]), _ptr(hp["out"]))
        hp["args"] = (_ptr(self.gamma_q), _ptr(self.gamma_k),
                      ctypes.c_float(self.eps), _ptr(self.cos), _ptr(self.sin), self.cos.shape[0],
                      _ptr(block_tables), block_tables.shape[1], _ptr(kp), _ptr(vp), kp.shape[0], b,
                      self.blocks_per_split, ctypes.c_float(SCALE), _ptr(self.part_ml), _ptr(self.part_o),
                      _ptr(self.counters), _ptr(self.dev_err))
        self._hp = hp

    def set_host_tables(self, block_tables: torch.Tensor) -> None:
        """Point the host-fed pipeline at another block table of the pipeline's
        shape (a scheduler that fills the next step's table while the current
        one is in use); the next step_host() reads it.  A table must stay alive
        and unchanged until the steps that read it have run."""
        hp = self._hp
        _need(block_tables, "block_tables", torch.int32, self.device, shape=hp["tables"].shape)
        args = list(hp["args"])
        args[6] = _ptr(block_tables)
        hp["args"] = tuple(args)
        hp["tables"] = block_tables

    def step_host(self, qkv_host: torch.Tensor, past_host: torch.Tensor, out_host: torch.Tensor,
                  stream: torch.cuda.Stream | None = None) -> None:
        """One decode step fed from pinned host memory (one C-ABI call): H2D of
        the qkv rows [B, 2048] and past lengths [B], the fused kernel on the
        current stream, D2H of the context into out_host [B, 16, 64].  When
        double-buffered, consecutive calls alternate two device slots, so
        uploads and downloads overlap the neighbouring steps' kernels.
        Asynchronous: the host buffers must stay alive and unchanged until
        join_host() and a synchronise of the stream; then out_host is valid."""
        hp = self._hp
        pinned = hp["pinned"]
        host = []
        for t, n, dt in ((qkv_host, hp["b"] * QKV_WIDTH, torch.bfloat16), (past_host, hp["b"], torch.int32),
                         (out_host, hp["b"] * HQ * D, torch.bfloat16)):
            if t.dtype != dt or t.numel() != n or not t.is_contiguous():
                raise ValueError("host buffers must be pinned, contiguous and of the pipeline's shape")
            # is_pinned() asks the CUDA host allocator (several us per call):
            # asked once per storage, so the rows of one pinned buffer (a
            # step's slice of it each call) are checked once.  A pinned block
            # stays pinned while the caching host allocator holds it.
            s = t.untyped_storage().data_ptr()
            if s not in pinned:
                if not t.is_pinned():
                    raise ValueError("host buffers must be pinned, contiguous and of the pipeline's shape")
                if len(pinned) >= 1024:
                    pinned.clear()
                pinned.add(s)
            host.append(t.data_ptr())
        if hp["double"]:
            rc = hp["call"](*host, *hp["bufs"], hp["slot"], *hp["args"], _stream(self.device, stream))
            hp["slot"] ^= 1
        else:
            rc = hp["call"](*host, *hp["bufs"], *hp["args"], _stream(self.device, stream))
        _lib.check(rc, "b2_decode_step_host2" if hp["double"] else "b2_decode_step_host")

    def join_host(self, stream: torch.cuda.Stream | None = None) -> None:
        """Make the stream wait for every context download issued by step_host
        (a no-op for the single-buffered pipeline, whose copies are in stream order)."""
        if self._hp["double"]:
            _lib.check(self._hp["join"](_stream(self.device, stream)), "b2_decode_step_host_join")

    def check(self) -> None:
        """Synchronise on the device error word; raise if any kernel flagged one."""
        word = int(self.dev_err.item())
        if word:
            self.dev_err.zero_()
            self.counters.zero_()   # an aborted fused step may leave counts behind
            raise RuntimeError("decode attention device error: " + "; ".join(_lib.decode_dev_err(word)))
