"""Drop-in operators with the reference's NPU operator signatures.

Each function keeps the name, argument order, buffer meaning and error
behaviour of the reference's IRON operator that the Python decode loop calls
(experiments/007_lfm25_npu_chat.py:160-196): the caller owns every buffer,
outputs are pre-allocated `Out` arguments written in place, nothing is
returned, an out-of-range length raises ValueError and a failed run raises
RuntimeError.  Buffers are CUDA bf16 tensors (flat, like the reference's
`iron.tensor`s); the math runs in libb2attn.so.

The reference's per-head cache formats are converted to and from the paged
pool around the kernels (a layout adapter).  Those formats are
copy-on-append by contract (`next_cache` is a new buffer holding the old
cache plus one row), so the adapter's O(L) copies are part of the
interface, not of the paged hot path (attention.PagedDecodeAttention), which
appends in place.

q/k in `qkv` are already normalised and rotated, as the reference's
attention_prefix leaves them (experiments/lfm25_attention_prefix_kernel.py),
so these operators append and attend without norm/RoPE.

Formats (bf16 element offsets):
  qkv                 [q 16x64 | k 8x64 | v 8x64]                   2048
  qkv_and_hidden      [q | k | v | hidden 1024]                     3072
  packed_tail_input   [hidden 1024 | context 16x64]                 2048
  cache (context/append)  8 heads x [K L x 64 | V L x 64]
  fixed64 cache       8 heads x [len, 0, K 64 x 64, V 64 x 64]
  chunked cache       blocks x 8 heads x [len, 0, K 64 x 64, V 64 x 64]
  first cache         8 heads x [k 64 | v 64]
"""
from __future__ import annotations

import torch

from . import _lib
from .attention import append_rope, combine, decode_attn

HQ, HKV, D, BLOCK = 16, 8, 64, 64
QKV, QKV_HIDDEN, PACKED = 2048, 3072, 2048
FIXED_CAP = 64
HEAD_FIXED = 2 + 2 * FIXED_CAP * D      # elements per head in the fixed64 / chunked formats


def _check(t: torch.Tensor, name: str, numel: int | None = None):
    if not isinstance(t, torch.Tensor) or t.dtype != torch.bfloat16 or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA bfloat16 tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if numel is not None and t.numel() != numel:
        raise ValueError(f"{name} must have {numel} elements, got {t.numel()}")


def _attend(qkv: torch.Tensor, keys: torch.Tensor, values: torch.Tensor):
    """Context of the qkv row's query over keys/values [8, L, 64] plus the
    row's own k, v (appended at L).  Returns (context [16, 64], pool K/V
    [nb, 8, 64, 64] holding the L + 1 rows)."""
    dev = qkv.device
    length = keys.shape[1]
    nb = (length + 1 + BLOCK - 1) // BLOCK
    pad = nb * BLOCK - length
    kp = torch.nn.functional.pad(keys, (0, 0, 0, pad)).reshape(HKV, nb, BLOCK, D).transpose(0, 1).contiguous()
    vp = torch.nn.functional.pad(values, (0, 0, 0, pad)).reshape(HKV, nb, BLOCK, D).transpose(0, 1).contiguous()
    table = torch.arange(nb, dtype=torch.int32, device=dev).reshape(1, nb)
    past = torch.tensor([length], dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    row = qkv[:QKV].reshape(1, QKV)
    q = row[:, : HQ * D].reshape(1, HQ, D).contiguous()
    append_rope(row.contiguous(), past, q_out=None, dev_err=err, mode=_lib.B2_STORE_KV,
                k_pool=kp, v_pool=vp, block_tables=table)
    ml = torch.empty(1, nb, HQ, 2, dtype=torch.float32, device=dev)
    po = torch.empty(1, nb, HQ, D, dtype=torch.float32, device=dev)
    seq = past + 1
    splits = decode_attn(q, kp, vp, table, seq, blocks_per_split=1, part_ml=ml, part_o=po, dev_err=err)
    ctx = torch.empty(1, HQ, D, dtype=torch.bfloat16, device=dev)
    combine(ml, po, splits, 1, seq_lens=seq, blocks_per_split=1, out=ctx)
    word = int(err.item())
    if word:
        raise RuntimeError("attention run failed: " + "; ".join(_lib.decode_dev_err(word)))
    return ctx[0], kp, vp


def _dense(kp: torch.Tensor, vp: torch.Tensor, length: int):
    nb = kp.shape[0]
    k = kp.transpose(0, 1).reshape(HKV, nb * BLOCK, D)[:, :length]
    v = vp.transpose(0, 1).reshape(HKV, nb * BLOCK, D)[:, :length]
    return k, v


def _split_cache(cache: torch.Tensor, length: int):
    c = cache.reshape(HKV, 2, length, D)
    return c[:, 0], c[:, 1]


def _write_cache(out: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    out.view(HKV, 2, k.shape[1], D).copy_(torch.stack([k, v], dim=1))


def _bf16_scalar(x: float, dev) -> torch.Tensor:
    return torch.tensor([x], dtype=torch.bfloat16, device=dev)


def _fixed_lengths(cache: torch.Tensor, heads: int) -> list[int]:
    lens = cache.view(-1, HEAD_FIXED)[:heads, 0].float().tolist()
    return [int(x) for x in lens]


# ----------------------------------------------------------------- operators

def append_attention_cache(qkv, prior_cache, next_cache) -> None:
    """experiments/lfm25_attention_append_cache_kernel.py:20-73: next_cache =
    prior_cache with the row's k, v appended to every head (bit-exact copy)."""
    _check(qkv, "qkv")
    if qkv.numel() < QKV:
        raise ValueError("qkv must hold at least 2048 elements")
    _check(prior_cache, "prior_cache")
    if prior_cache.numel() % (HKV * 2 * D):
        raise ValueError("prior_cache is not 8 heads x [K L x 64 | V L x 64]")
    length = prior_cache.numel() // (HKV * 2 * D)
    _check(next_cache, "next_cache", HKV * 2 * (length + 1) * D)
    keys, values = _split_cache(prior_cache, length)
    dev = qkv.device
    nb = (length + 1 + BLOCK - 1) // BLOCK
    pad = nb * BLOCK - length
    kp = torch.nn.functional.pad(keys, (0, 0, 0, pad)).reshape(HKV, nb, BLOCK, D).transpose(0, 1).contiguous()
    vp = torch.nn.functional.pad(values, (0, 0, 0, pad)).reshape(HKV, nb, BLOCK, D).transpose(0, 1).contiguous()
    table = torch.arange(nb, dtype=torch.int32, device=dev).reshape(1, nb)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    append_rope(qkv.reshape(-1)[:QKV].reshape(1, QKV).contiguous(),
                torch.tensor([length], dtype=torch.int32, device=dev), q_out=None, dev_err=err,
                mode=_lib.B2_STORE_KV, k_pool=kp, v_pool=vp, block_tables=table)
    if int(err.item()):
        raise RuntimeError("append run failed")
    k, v = _dense(kp, vp, length + 1)
    _write_cache(next_cache, k, v)


def attention_context(qkv, past_cache, context) -> None:
    """experiments/lfm25_attention_context_kernel.py:20-72: context [16 x 64]
    of the row's query over the past cache plus the row's own k, v."""
    _check(qkv, "qkv")
    if qkv.numel() < QKV:
        raise ValueError("qkv must hold at least 2048 elements")
    _check(past_cache, "past_cache")
    if past_cache.numel() % (HKV * 2 * D):
        raise ValueError("past_cache is not 8 heads x [K L x 64 | V L x 64]")
    length = past_cache.numel() // (HKV * 2 * D)
    _check(context, "context", HQ * D)
    keys, values = _split_cache(past_cache, length)
    ctx, _, _ = _attend(qkv.reshape(-1), keys, values)
    context.view(HQ, D).copy_(ctx)


def attention_context_cache(qkv_and_hidden, past_cache, packed_tail_input, next_cache, *,
                            past_length: int = 21) -> None:
    """experiments/lfm25_attention_context_cache_kernel.py:16-106: packed tail
    [hidden | context] and next_cache (past + the row's k, v).  The reference
    compiles one program per past_length and accepts 1-95; any past_length >= 1
    that matches the buffers is accepted here, others raise ValueError."""
    if past_length < 1:
        raise ValueError("past_length must be >= 1")
    _check(qkv_and_hidden, "qkv_and_hidden", QKV_HIDDEN)
    _check(past_cache, "past_cache", HKV * 2 * past_length * D)
    _check(packed_tail_input, "packed_tail_input", PACKED)
    _check(next_cache, "next_cache", HKV * 2 * (past_length + 1) * D)
    keys, values = _split_cache(past_cache, past_length)
    ctx, kp, vp = _attend(qkv_and_hidden, keys, values)
    packed_tail_input[:1024].copy_(qkv_and_hidden[2048:3072])
    packed_tail_input[1024:].copy_(ctx.reshape(-1))
    k, v = _dense(kp, vp, past_length + 1)
    _write_cache(next_cache, k, v)


def attention_first_context(qkv_and_hidden, packed_tail_input, first_cache) -> None:
    """experiments/lfm25_attention_first_context_kernel.py:16-49 (kernel
    experiments/kernels/lfm25_attention_first_context.cc:4-22): position 0,
    where softmax over one key returns its value; the cache is [k | v] per head."""
    _check(qkv_and_hidden, "qkv_and_hidden", QKV_HIDDEN)
    _check(packed_tail_input, "packed_tail_input", PACKED)
    _check(first_cache, "first_cache", HKV * 2 * D)
    dev = qkv_and_hidden.device
    empty = torch.empty(HKV, 0, D, dtype=torch.bfloat16, device=dev)
    ctx, kp, vp = _attend(qkv_and_hidden, empty, empty)
    packed_tail_input[:1024].copy_(qkv_and_hidden[2048:3072])
    packed_tail_input[1024:].copy_(ctx.reshape(-1))
    first_cache.view(HKV, 2, D).copy_(torch.stack([kp[0, :, 0], vp[0, :, 0]], dim=1))


def attention_context_fixed64(qkv_and_hidden, past_cache, packed_tail_input, next_cache) -> None:
    """experiments/lfm25_attention_fixed64_cache_kernel.py:81-136 (kernel
    lfm25_attention_fixed64_head, experiments/kernels/lfm25_attention_fixed64_head.cc:40-97):
    fixed 64-slot cache whose element 0 per head is the length (bf16)."""
    _check(qkv_and_hidden, "qkv_and_hidden", QKV_HIDDEN)
    _check(past_cache, "past_cache", HKV * HEAD_FIXED)
    _check(packed_tail_input, "packed_tail_input", PACKED)
    _check(next_cache, "next_cache", HKV * HEAD_FIXED)
    lens = _fixed_lengths(past_cache, HKV)
    length = lens[0]
    if any(n != length for n in lens) or not 1 <= length < FIXED_CAP:
        raise ValueError(f"fixed64 cache length must be 1-63 and equal across heads, got {lens}")
    heads = past_cache.view(HKV, HEAD_FIXED)
    keys = heads[:, 2: 2 + length * D].reshape(HKV, length, D)
    values = heads[:, 2 + FIXED_CAP * D: 2 + FIXED_CAP * D + length * D].reshape(HKV, length, D)
    ctx, kp, vp = _attend(qkv_and_hidden, keys, values)
    packed_tail_input[:1024].copy_(qkv_and_hidden[2048:3072])
    packed_tail_input[1024:].copy_(ctx.reshape(-1))
    out = next_cache.view(HKV, HEAD_FIXED)
    out.copy_(past_cache.view(HKV, HEAD_FIXED))
    k, v = _dense(kp, vp, length + 1)
    out[:, 0] = _bf16_scalar(float(length + 1), qkv_and_hidden.device)
    out[:, 2 + length * D: 2 + (length + 1) * D] = k[:, length]
    out[:, 2 + FIXED_CAP * D + length * D: 2 + FIXED_CAP * D + (length + 1) * D] = v[:, length]


def attention_first_fixed64(qkv_and_hidden, packed_tail_input, first_cache) -> None:
    """experiments/lfm25_attention_fixed64_cache_kernel.py:30-78 (kernel
    lfm25_attention_fixed64_first_head, experiments/kernels/lfm25_attention_fixed64_head.cc:25-38):
    position 0 into an empty fixed64 cache (length 1)."""
    _check(qkv_and_hidden, "qkv_and_hidden", QKV_HIDDEN)
    _check(packed_tail_input, "packed_tail_input", PACKED)
    _check(first_cache, "first_cache", HKV * HEAD_FIXED)
    dev = qkv_and_hidden.device
    empty = torch.empty(HKV, 0, D, dtype=torch.bfloat16, device=dev)
    ctx, kp, vp = _attend(qkv_and_hidden, empty, empty)
    packed_tail_input[:1024].copy_(qkv_and_hidden[2048:3072])
    packed_tail_input[1024:].copy_(ctx.reshape(-1))
    out = first_cache.view(HKV, HEAD_FIXED)
    out.zero_()
    out[:, 0] = _bf16_scalar(1.0, dev)
    out[:, 2: 2 + D] = kp[0, :, 0]
    out[:, 2 + FIXED_CAP * D: 2 + FIXED_CAP * D + D] = vp[0, :, 0]


def attention_context_chunked(qkv_and_hidden, past_cache, packed_tail_input, next_cache, *,
                              block_count: int = 1) -> None:
    """experiments/lfm25_attention_chunked_cache_kernel.py:21-89 (kernel
    lfm25_attention_chunked_head, experiments/kernels/lfm25_attention_chunked_head.cc:26-91):
    block_count 64-token blocks, each (block, head) = [len, 0, K 64 x 64, V 64 x 64];
    the new k, v go into the last block.  The reference's 64-block (4K) limit
    is an NPU memory limit and is not imposed; block_count < 1 raises ValueError."""
    if block_count < 1:
        raise ValueError("block_count must be >= 1")
    size = block_count * HKV * HEAD_FIXED
    _check(qkv_and_hidden, "qkv_and_hidden", QKV_HIDDEN)
    _check(past_cache, "past_cache", size)
    _check(packed_tail_input, "packed_tail_input", PACKED)
    _check(next_cache, "next_cache", size)
    blocks = past_cache.view(block_count, HKV, HEAD_FIXED)
    lens = blocks[:, :, 0].float().cpu()
    if not bool((lens == lens[:, :1]).all()):
        raise ValueError("chunked cache lengths differ across heads")
    per_block = [int(x) for x in lens[:, 0].tolist()]
    if any(n != FIXED_CAP for n in per_block[:-1]) or not 0 <= per_block[-1] < FIXED_CAP:
        raise ValueError(f"chunked cache needs full blocks and room in the last one, got {per_block}")
    length = FIXED_CAP * (block_count - 1) + per_block[-1]
    keys = blocks[:, :, 2: 2 + FIXED_CAP * D].reshape(block_count, HKV, FIXED_CAP, D)
    values = blocks[:, :, 2 + FIXED_CAP * D:].reshape(block_count, HKV, FIXED_CAP, D)
    keys = keys.transpose(0, 1).reshape(HKV, block_count * FIXED_CAP, D)[:, :length]
    values = values.transpose(0, 1).reshape(HKV, block_count * FIXED_CAP, D)[:, :length]
    ctx, kp, vp = _attend(qkv_and_hidden, keys, values)
    packed_tail_input[:1024].copy_(qkv_and_hidden[2048:3072])
    packed_tail_input[1024:].copy_(ctx.reshape(-1))
    out = next_cache.view(block_count, HKV, HEAD_FIXED)
    out.copy_(blocks)
    k, v = _dense(kp, vp, length + 1)
    slot = per_block[-1]
    last = out[block_count - 1]
    last[:, 0] = _bf16_scalar(float(slot + 1), qkv_and_hidden.device)
    last[:, 2 + slot * D: 2 + (slot + 1) * D] = k[:, length]
    last[:, 2 + FIXED_CAP * D + slot * D: 2 + FIXED_CAP * D + (slot + 1) * D] = v[:, length]
