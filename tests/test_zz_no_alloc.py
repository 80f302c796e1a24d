"""The allocation-free decode entry point, b2_decode_attn_noalloc.

Some callers hold device pointers but cannot allocate device memory
themselves: a host in another language bound only to the C ABI, with no CUDA
allocator, or an embedder whose device memory is all committed to another
framework.  For them the library keeps the partial softmax states in its own
static device array (B2_NOALLOC_MAX_PARTS sequence-splits per GPU).

These tests call the entry point through the C ABI (ctypes) twice in a row,
with different batches, and compare each output with the existing path
(b2_decode_attn into caller buffers + b2_combine) within the attention
tolerance the other GPU tests use.  The file is named so that pytest collects
it last.
"""
import ctypes

import pytest
import torch

from conftest import load_pkg
from oracle import lfm2_attention as orc

pytestmark = pytest.mark.gpu

ATOL = 2e-2
RTOL = 1e-2


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _batch(lengths, seed, dev):
    pc = load_pkg("paged_cache")
    cache = pc.PagedKVCache(sum(pc.blocks_for(n) for n in lengths) + 2, max(lengths), device=dev,
                            shuffle_seed=seed, fill=float("nan"))
    for i, n in enumerate(lengths):
        cache.add_sequence(n, capacity=n)
        k, v = orc.past_cache(seed * 100 + i, n)
        cache.write_dense(0, i, k[0], v[0])
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(len(lengths), 16, 64, generator=g).to(torch.bfloat16).to(dev)
    seq = torch.tensor(lengths, dtype=torch.int32, device=dev)
    return cache, q, seq


def _existing(cache, q, seq, bps):
    attn = load_pkg("attention")
    b = q.shape[0]
    tables = cache.block_tables()
    splits = attn.num_splits_for(tables.shape[1], bps)
    ml = torch.empty(b, splits, 16, 2, dtype=torch.float32, device=q.device)
    po = torch.empty(b, splits, 16, 64, dtype=torch.float32, device=q.device)
    err = torch.zeros(1, dtype=torch.int32, device=q.device)
    kp, vp = cache.pool(0)
    attn.decode_attn(q, kp, vp, tables, seq, blocks_per_split=bps, part_ml=ml, part_o=po, dev_err=err)
    out = torch.empty(b, 16, 64, dtype=torch.bfloat16, device=q.device)
    attn.combine(ml, po, splits, b, seq_lens=seq, blocks_per_split=bps, out=out)
    torch.cuda.synchronize()
    assert err.item() == 0
    return out


def _noalloc(cache, q, seq, bps):
    lib = load_pkg("_lib")
    b = q.shape[0]
    tables = cache.block_tables()
    kp, vp = cache.pool(0)
    out = torch.full((b, 16, 64), float("nan"), dtype=torch.bfloat16, device=q.device)
    err = torch.zeros(1, dtype=torch.int32, device=q.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)
    rc = lib.load().b2_decode_attn_noalloc(_ptr(q), _ptr(kp), _ptr(vp), kp.shape[0], _ptr(tables),
                                           tables.shape[1], _ptr(seq), b, bps, ctypes.c_float(0.125),
                                           _ptr(out), _ptr(err), stream)
    lib.check(rc, "b2_decode_attn_noalloc")
    torch.cuda.synchronize()
    assert err.item() == 0
    return out


def test_noalloc_matches_existing_entry_point_twice(cuda):
    """Two calls in a row; the second reuses the static array the first left behind."""
    cases = [([1, 64, 65, 700, 3000], 41, 2), ([5000, 17, 129, 2048], 42, 3)]
    for lengths, seed, bps in cases:
        cache, q, seq = _batch(lengths, seed, cuda)
        ref = _existing(cache, q, seq, bps).float().cpu()
        got = _noalloc(cache, q, seq, bps).float().cpu()
        assert torch.isfinite(got).all()
        err = (got - ref).abs().max().item()
        rel = ((got - ref).norm() / ref.norm()).item()
        assert err <= ATOL and rel <= RTOL, f"lengths {lengths}: max-abs {err}, rel {rel}"


def test_noalloc_rejects_sizes_beyond_the_static_array(cuda):
    lib = load_pkg("_lib")
    cache, q, seq = _batch([64], 43, cuda)
    tables = cache.block_tables()
    kp, vp = cache.pool(0)
    out = torch.empty(1, 16, 64, dtype=torch.bfloat16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    too_many = lib.B2_NOALLOC_MAX_PARTS + 1   # batch x 1 split > limit
    rc = lib.load().b2_decode_attn_noalloc(_ptr(q), _ptr(kp), _ptr(vp), kp.shape[0], _ptr(tables),
                                           tables.shape[1], _ptr(seq), too_many, 1, ctypes.c_float(0.125),
                                           _ptr(out), _ptr(err), None)
    assert rc == lib.B2_ERR_ARG
    assert "B2_NOALLOC_MAX_PARTS" in lib.last_error()
