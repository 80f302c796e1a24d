"""Batched-prompt (prefill) attention on the tcgen05 tensor cores, against
the reference's CPU path for a chunk of tokens after a cached prefix
(transformers Lfm2Attention with the causal mask of a cached prefix; golden
fixtures tests/golden/lfm2_prefill_*.npz and the oracle for ragged batches).
Tolerance as for decode: max-abs 2e-2, relative L2 1e-2."""
import pathlib

import numpy as np
import pytest
import torch

from conftest import load_pkg
from oracle import lfm2_attention as orc
from test_kernels_gpu import build_batch, check_close, rand_qkv, ulp_diff

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def _run_prefill(cuda, cache, qkv, past, chunk, gq, gk, blocks_per_split=None):
    attn = load_pkg("attention")
    rope = load_pkg("rope")
    cos, sin = rope.rope_table(4096, device=cuda)
    kp, vp = cache.pool(0)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = attn.prefill(qkv.to(cuda), torch.tensor(past, dtype=torch.int32, device=cuda), k_pool=kp, v_pool=vp,
                       block_tables=cache.block_tables(), gamma_q=gq.to(cuda), gamma_k=gk.to(cuda), cos=cos,
                       sin=sin, dev_err=err, blocks_per_split=blocks_per_split,
                       chunk_lens=None if chunk is None else torch.tensor(chunk, dtype=torch.int32, device=cuda))
    torch.cuda.synchronize()
    assert err.item() == 0
    return out


def assert_k_exact(kd: torch.Tensor, k_ref: torch.Tensor) -> None:
    """Appended k (RMSNorm + RoPE in the append kernel) against the oracle:
    bit-identical (the squares are summed in torch's CPU order)."""
    ulp = ulp_diff(kd, k_ref)
    assert (ulp == 0).all(), f"{(ulp != 0).sum()} of {ulp.size} elements differ (max {ulp.max()} ulps)"


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("lfm2_prefill_*.npz")), ids=lambda p: p.stem)
def test_prefill_matches_hf_golden(cuda, path):
    f = dict(np.load(path))
    past, t = int(f["past"]), int(f["tokens"])
    w = orc.attention_weights(int(f["weight_seed"]))
    k, v = orc.past_cache(3000 + past, past)
    cache, _ = build_batch([past], cuda, seed=0, capacity=past + t + 1)
    cache.write_dense(0, 0, k[0], v[0])
    qkv = orc.from_bits(f["qkv"]).reshape(1, t, -1)
    out = _run_prefill(cuda, cache, qkv, [past], None, w["q_gamma"], w["k_gamma"])
    check_close(out[0], orc.from_bits(f["context"]).reshape(t, 16, 64), path.stem)
    # the chunk's k/v were appended bit-exactly
    _, k_all, v_all = orc.prefill_step(qkv[0], k[0], v[0], past, w["q_gamma"], w["k_gamma"])
    kd, vd = cache.read_dense(0, 0, past + t)
    assert torch.equal(vd.cpu(), v_all)
    assert_k_exact(kd, k_all)


def test_prefill_ragged_batch(cuda):
    past = [0, 63, 64, 500, 7]
    chunk = [1, 5, 64, 100, 129]
    tmax = 130
    w = orc.attention_weights(0)
    cache, hist = build_batch(past, cuda, seed=21, capacity=max(p + c for p, c in zip(past, chunk)) + 1)
    qkv = torch.stack([rand_qkv(tmax, 700 + i) for i in range(len(past))])     # [B, tmax, 2048]
    out = _run_prefill(cuda, cache, qkv, past, chunk, w["q_gamma"], w["k_gamma"])
    for i, (p, c) in enumerate(zip(past, chunk)):
        ctx, _, _ = orc.prefill_step(qkv[i, :c], hist[i][0], hist[i][1], p, w["q_gamma"], w["k_gamma"])
        check_close(out[i, :c], ctx, f"seq {i} past {p} chunk {c}")


@pytest.mark.parametrize("bps", [1, 3, 16])
def test_prefill_split_keys_ragged(cuda, bps):
    """Keys split over CTAs (b2_prefill_attn_split) for short chunks: against
    the oracle, with splits past a sequence's keys and chunks shorter than the
    tile; rows past a chunk come out 0."""
    past = [0, 63, 64, 500, 7, 2000]
    chunk = [1, 5, 16, 3, 32, 4]
    tmax = 32
    w = orc.attention_weights(0)
    cache, hist = build_batch(past, cuda, seed=23, capacity=max(p + c for p, c in zip(past, chunk)) + 1)
    qkv = torch.stack([rand_qkv(tmax, 900 + i) for i in range(len(past))])     # [B, tmax, 2048]
    out = _run_prefill(cuda, cache, qkv, past, chunk, w["q_gamma"], w["k_gamma"], blocks_per_split=bps)
    for i, (p, c) in enumerate(zip(past, chunk)):
        ctx, _, _ = orc.prefill_step(qkv[i, :c], hist[i][0], hist[i][1], p, w["q_gamma"], w["k_gamma"])
        check_close(out[i, :c], ctx, f"seq {i} past {p} chunk {c} bps {bps}")
        assert not out[i, c:].float().abs().any(), f"seq {i}: rows past the chunk not zero"


def test_prefill_split_matches_unsplit(cuda):
    """The same chunk with and without the key split: contexts within the
    attention tolerance of each other (fp32 merges in another order)."""
    past = [3000, 100, 4000]
    w = orc.attention_weights(0)
    outs = []
    for bps in (0, 7):
        cache, _ = build_batch(past, cuda, seed=24, capacity=max(past) + 9)
        qkv = torch.stack([rand_qkv(8, 950 + i) for i in range(len(past))])
        outs.append(_run_prefill(cuda, cache, qkv, past, None, w["q_gamma"], w["k_gamma"], blocks_per_split=bps))
    check_close(outs[1], outs[0].float().cpu(), "split vs unsplit")


def test_prefill_then_decode(cuda):
    """A 70-token prompt through the tcgen05 prefill, then three decode steps
    through the fused decode kernel on the same paged cache."""
    attn = load_pkg("attention")
    w = orc.attention_weights(0)
    cache, _ = build_batch([0], cuda, seed=22, capacity=128)
    prompt = rand_qkv(70, 800)[None]
    _run_prefill(cuda, cache, prompt, [0], None, w["q_gamma"], w["k_gamma"])
    _, k_hist, v_hist = orc.prefill_step(prompt[0], torch.zeros(8, 0, 64, dtype=torch.bfloat16),
                                         torch.zeros(8, 0, 64, dtype=torch.bfloat16), 0, w["q_gamma"], w["k_gamma"])
    kd, vd = cache.read_dense(0, 0, 70)
    assert_k_exact(kd, k_hist)
    assert torch.equal(vd.cpu(), v_hist)
    runner = attn.PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], 1, 256, blocks_per_split=1)
    for step in range(3):
        raw = rand_qkv(1, 900 + step)
        past = torch.tensor([70 + step], dtype=torch.int32, device=cuda)
        out = runner.step(0, raw.to(cuda), past, past + 1, cache.block_tables())
        torch.cuda.synchronize()
        runner.check()
        ctx, k_hist, v_hist, _ = orc.decode_step(raw[0], k_hist, v_hist, 70 + step, w["q_gamma"], w["k_gamma"])
        check_close(out[0], ctx, f"decode step {step} after prefill")
        kd, vd = cache.read_dense(0, 0, 71 + step)
        assert torch.equal(kd.cpu(), k_hist) and torch.equal(vd.cpu(), v_hist), f"cache after step {step}"
