"""Host-side checks of the drop-in operators (ryzenai-npu-lab_b200/operators.py),
which raise ValueError like the reference's operators do for an out-of-range
length (experiments/lfm25_attention_context_cache_kernel.py:25-26,
experiments/lfm25_attention_chunked_cache_kernel.py:25-26) before any work
is queued; no GPU is needed for these."""
import pytest
import torch

from conftest import load_pkg

BF = torch.bfloat16


def test_out_of_range_lengths_raise_value_error():
    ops = load_pkg("operators")
    t = torch.zeros(8, dtype=BF)
    with pytest.raises(ValueError, match="past_length"):
        ops.attention_context_cache(t, t, t, t, past_length=0)
    with pytest.raises(ValueError, match="block_count"):
        ops.attention_context_chunked(t, t, t, t, block_count=0)


def test_buffers_must_be_cuda_bf16_of_the_right_size():
    ops = load_pkg("operators")
    cpu = torch.zeros(3072, dtype=BF)
    with pytest.raises(ValueError, match="CUDA bfloat16"):
        ops.attention_context_cache(cpu, torch.zeros(8 * 2 * 21 * 64, dtype=BF), torch.zeros(2048, dtype=BF),
                                    torch.zeros(8 * 2 * 22 * 64, dtype=BF), past_length=21)
    with pytest.raises(ValueError, match="CUDA bfloat16"):
        ops.attention_context_cache(cpu.float(), cpu, cpu, cpu, past_length=21)
    with pytest.raises(ValueError):
        ops.append_attention_cache(torch.zeros(100, dtype=BF), cpu, cpu)


@pytest.mark.parametrize("length", [1, 21, 64, 95])
def test_per_head_cache_formats_match_the_reference_layouts(length):
    """The operators' host-side format helpers read and write the reference's
    per-head cache layouts exactly as the oracle restates them: [K L x 64 |
    V L x 64] per head (lfm25_attention_append_cache.cc:5-39) and the fixed64
    / chunked headers holding the length as bf16 in element 0 of each head
    (lfm25_attention_fixed64_head.cc:25-57, lfm25_attention_chunked_head.cc:26-47)."""
    import numpy as np
    from oracle import lfm2_attention as orc
    ops = load_pkg("operators")
    g = torch.Generator().manual_seed(length)
    k = torch.randn(8, length, 64, generator=g).to(BF)
    v = torch.randn(8, length, 64, generator=g).to(BF)
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16).reshape(-1)
    # [K | V] per head: what _write_cache writes is the layout the reference's append grows
    cache = torch.empty(8 * 2 * length * 64, dtype=BF)
    ops._write_cache(cache, k, v)
    prior = np.stack([bits(k).reshape(8, length, 64), bits(v).reshape(8, length, 64)], axis=1).reshape(-1)
    assert np.array_equal(bits(cache), prior)
    qkv = bits(torch.randn(2048, generator=g).to(BF))
    grown = orc.ref_append_cache(qkv, prior)
    kk, vv = ops._split_cache(torch.from_numpy(grown.view(np.int16).copy()).view(BF), length + 1)
    assert torch.equal(kk[:, :length], k) and torch.equal(vv[:, :length], v)
    assert np.array_equal(bits(kk[:, length]), qkv[1024:1536].reshape(8, 64).reshape(-1))
    # fixed64 and chunked headers: the length each head holds
    if length <= 64:
        fixed = orc.ref_fixed64_cache(bits(k).reshape(8, length, 64), bits(v).reshape(8, length, 64))
        assert ops._fixed_lengths(torch.from_numpy(fixed.view(np.int16).copy()).view(BF), 8) == [length] * 8
    blocks = (length + 63) // 64 + 1
    chunked = orc.ref_chunked_cache(bits(k).reshape(8, length, 64), bits(v).reshape(8, length, 64), blocks)
    per_block = torch.from_numpy(chunked.view(np.int16).copy()).view(BF).view(blocks, -1)
    got = [ops._fixed_lengths(per_block[j], 8)[0] for j in range(blocks)]
    assert got == [max(0, min(64, length - 64 * j)) for j in range(blocks)]
