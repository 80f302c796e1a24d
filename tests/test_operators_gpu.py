"""Drop-in operators with the reference's NPU signatures, checked the way the
reference's hardware validation scripts check them
(006_lfm25_npu_attention_context.py:82-87: new key/value and next cache
bit-exact, context close; 006_lfm25_npu_attention_two_tokens.py:84-87: two
chained tokens; 006_lfm25_npu_attention_first.py:69-70: position 0), with the
CPU oracle in place of the missing fixtures."""
import numpy as np
import pytest
import torch

from conftest import load_pkg
from oracle import lfm2_attention as orc
from test_kernels_gpu import check_close

pytestmark = pytest.mark.gpu


def ops():
    return load_pkg("operators")


def qkv_hidden(seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(3072, generator=g).to(torch.bfloat16)


def past(seed, length):
    k, v = orc.past_cache(seed, length)
    return k[0], v[0]


def oracle_ctx(row, keys, values):
    """Context of row's (already rotated) q over keys/values + the row's k, v."""
    q, k, v = orc.split_qkv(row[:2048].reshape(1, -1))
    kk = torch.cat([keys, k[0][:, None]], dim=1)
    vv = torch.cat([values, v[0][:, None]], dim=1)
    return orc.attend(q[:, :, None, :], kk[None], vv[None], "sdpa").reshape(16, 64), kk, vv


def per_head_cache(keys, values):
    return torch.stack([keys, values], dim=1).reshape(-1)


@pytest.mark.parametrize("length", [1, 21, 63, 64, 200])
def test_append_attention_cache_bit_exact(cuda, length):
    row = qkv_hidden(length)[:2048]
    keys, values = past(length, length)
    prior = per_head_cache(keys, values)
    nxt = torch.empty(8 * 2 * (length + 1) * 64, dtype=torch.bfloat16, device=cuda)
    ops().append_attention_cache(row.to(cuda), prior.to(cuda), nxt)
    ref = orc.ref_append_cache(orc.bits(row), orc.bits(prior))
    assert np.array_equal(orc.bits(nxt.cpu()), ref)


@pytest.mark.parametrize("length", [1, 21, 95, 300])
def test_attention_context_cache(cuda, length):
    row = qkv_hidden(100 + length)
    keys, values = past(200 + length, length)
    prior = per_head_cache(keys, values)
    packed = torch.empty(2048, dtype=torch.bfloat16, device=cuda)
    nxt = torch.empty(8 * 2 * (length + 1) * 64, dtype=torch.bfloat16, device=cuda)
    ops().attention_context_cache(row.to(cuda), prior.to(cuda), packed, nxt, past_length=length)
    ctx_ref, _, _ = oracle_ctx(row, keys, values)
    assert torch.equal(packed[:1024].cpu(), row[2048:])
    check_close(packed[1024:].reshape(16, 64), ctx_ref, f"context L={length}")
    assert np.array_equal(orc.bits(nxt.cpu()), orc.ref_append_cache(orc.bits(row), orc.bits(prior)))
    ctx = torch.empty(1024, dtype=torch.bfloat16, device=cuda)
    ops().attention_context(row[:2048].to(cuda), prior.to(cuda), ctx)
    assert torch.equal(ctx.cpu(), packed[1024:].cpu())


def test_two_chained_tokens(cuda):
    length = 21
    keys, values = past(7, length)
    cache = per_head_cache(keys, values).to(cuda)
    rows = [qkv_hidden(8), qkv_hidden(9)]
    for t, row in enumerate(rows):
        packed = torch.empty(2048, dtype=torch.bfloat16, device=cuda)
        nxt = torch.empty(8 * 2 * (length + t + 1) * 64, dtype=torch.bfloat16, device=cuda)
        ops().attention_context_cache(row.to(cuda), cache, packed, nxt, past_length=length + t)
        ctx_ref, keys, values = oracle_ctx(row, keys, values)
        check_close(packed[1024:].reshape(16, 64), ctx_ref, f"token {t}")
        assert torch.equal(nxt.cpu(), per_head_cache(keys, values))
        cache = nxt


def test_first_context_is_value(cuda):
    row = qkv_hidden(11)
    packed = torch.empty(2048, dtype=torch.bfloat16, device=cuda)
    first = torch.empty(1024, dtype=torch.bfloat16, device=cuda)
    ops().attention_first_context(row.to(cuda), packed, first)
    _, k, v = orc.split_qkv(row[:2048].reshape(1, -1))
    assert torch.equal(first.cpu().reshape(8, 2, 64), torch.stack([k[0], v[0]], dim=1))
    assert torch.equal(packed[1024:].cpu().reshape(8, 2, 64), torch.stack([v[0], v[0]], dim=1))
    assert torch.equal(packed[:1024].cpu(), row[2048:])


def test_fixed64_first_then_context(cuda):
    row0, row1 = qkv_hidden(12), qkv_hidden(13)
    packed = torch.empty(2048, dtype=torch.bfloat16, device=cuda)
    c0 = torch.empty(8 * (2 + 2 * 64 * 64), dtype=torch.bfloat16, device=cuda)
    ops().attention_first_fixed64(row0.to(cuda), packed, c0)
    _, k0, v0 = orc.split_qkv(row0[:2048].reshape(1, -1))
    assert np.array_equal(orc.bits(c0.cpu()), orc.ref_fixed64_cache(orc.bits(k0[0][:, None]), orc.bits(v0[0][:, None])))
    c1 = torch.empty_like(c0)
    ops().attention_context_fixed64(row1.to(cuda), c0, packed, c1)
    ctx_ref, kk, vv = oracle_ctx(row1, k0[0][:, None], v0[0][:, None])
    check_close(packed[1024:].reshape(16, 64), ctx_ref, "fixed64 context")
    assert np.array_equal(orc.bits(c1.cpu()), orc.ref_fixed64_cache(orc.bits(kk), orc.bits(vv)))


def test_fixed64_full_cache_rejected(cuda):
    keys, values = past(14, 64)
    full = torch.from_numpy(orc.ref_fixed64_cache(orc.bits(keys), orc.bits(values)).view(np.int16)).view(torch.bfloat16)
    packed = torch.empty(2048, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        ops().attention_context_fixed64(qkv_hidden(15).to(cuda), full.to(cuda), packed, torch.empty_like(full, device=cuda))


@pytest.mark.parametrize("length,blocks", [(1, 1), (63, 1), (64, 2), (100, 2), (4095, 64), (5000, 79)])
def test_chunked(cuda, length, blocks):
    row = qkv_hidden(300 + length)
    keys, values = past(400 + length, length)
    prior = orc.ref_chunked_cache(orc.bits(keys), orc.bits(values), blocks)
    prior_t = torch.from_numpy(prior.view(np.int16)).view(torch.bfloat16).to(cuda)
    packed = torch.empty(2048, dtype=torch.bfloat16, device=cuda)
    nxt = torch.empty_like(prior_t)
    ops().attention_context_chunked(row.to(cuda), prior_t, packed, nxt, block_count=blocks)
    ctx_ref, kk, vv = oracle_ctx(row, keys, values)
    check_close(packed[1024:].reshape(16, 64), ctx_ref, f"chunked L={length}")
    assert np.array_equal(orc.bits(nxt.cpu()), orc.ref_chunked_cache(orc.bits(kk), orc.bits(vv), blocks))


def test_operator_errors(cuda):
    row = qkv_hidden(16).to(cuda)
    packed = torch.empty(2048, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        ops().attention_context_cache(row, torch.empty(10, dtype=torch.bfloat16, device=cuda), packed,
                                      torch.empty(10, dtype=torch.bfloat16, device=cuda), past_length=0)
    with pytest.raises(ValueError):
        ops().attention_context_chunked(row, torch.empty(10, dtype=torch.bfloat16, device=cuda), packed,
                                        torch.empty(10, dtype=torch.bfloat16, device=cuda), block_count=0)
    with pytest.raises(ValueError):
        ops().attention_context(row.float(), torch.empty(8 * 128, dtype=torch.bfloat16, device=cuda),
                                torch.empty(1024, dtype=torch.bfloat16, device=cuda))
