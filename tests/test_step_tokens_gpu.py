"""The fused decode step with 2-4 new tokens per sequence
(b2_decode_step_tokens: a prompt chunk, or the reference's x8p engine's
4-token batches) against the reference's CPU path for a chunk of tokens after
a cached prefix (transformers Lfm2Attention with the causal mask of a cached
prefix, restated in oracle.prefill_step): contexts within the attention
tolerance (max-abs 2e-2, relative L2 1e-2), the appended k/v and the rotated
q bit-exact.  Positions cross block boundaries (63 / 64 / 127 ...), chunks are
ragged, and the keys are split into several items merged in the kernel."""
import pytest
import torch

from conftest import load_pkg
from oracle import lfm2_attention as orc
from test_kernels_gpu import build_batch, check_close, rand_qkv, ulp_diff

pytestmark = pytest.mark.gpu


def _run(cuda, past, tokens, chunk=None, bps=None, seed=0, capacity=None, qkv=None, max_ctas=0):
    attn = load_pkg("attention")
    rope = load_pkg("rope")
    w = orc.attention_weights(seed)
    b = len(past)
    cap = capacity or (max(past) + tokens + 1)
    cache, hist = build_batch(past, cuda, seed=40 + seed, capacity=cap)
    if qkv is None:
        qkv = torch.stack([rand_qkv(tokens, 900 + 7 * i + seed) for i in range(b)])   # [B, T, 2048]
    cos, sin = rope.rope_table(cap + 8, device=cuda)
    kp, vp = cache.pool(0)
    out = torch.full((b, tokens, 16, 64), 7.0, dtype=torch.bfloat16, device=cuda)
    q_out = torch.empty(b, tokens, 16, 64, dtype=torch.bfloat16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    counters = torch.zeros(2 + 8 * b, dtype=torch.int32, device=cuda)
    splits = attn.decode_step_tokens(
        qkv.to(cuda), torch.tensor(past, dtype=torch.int32, device=cuda), k_pool=kp, v_pool=vp,
        block_tables=cache.block_tables(), out=out, counters=counters, dev_err=err, blocks_per_split=bps,
        gamma_q=w["q_gamma"].to(cuda), gamma_k=w["k_gamma"].to(cuda), cos=cos, sin=sin, q_out=q_out,
        chunk_lens=None if chunk is None else torch.tensor(chunk, dtype=torch.int32, device=cuda), max_ctas=max_ctas)
    torch.cuda.synchronize()
    assert err.item() == 0
    assert int(counters.abs().sum().item()) == 0          # the kernel leaves its counters zero
    return w, cache, hist, qkv, out, q_out, splits


def _check(w, cache, hist, qkv, out, q_out, past, chunks, what):
    for i, (p, c) in enumerate(zip(past, chunks)):
        ctx, k_all, v_all = orc.prefill_step(qkv[i, :c], hist[i][0], hist[i][1], p, w["q_gamma"], w["k_gamma"])
        check_close(out[i, :c], ctx, f"{what}: seq {i} past {p} chunk {c}")
        kd, vd = cache.read_dense(0, i, p + c)
        assert torch.equal(vd.cpu(), v_all), f"{what}: seq {i} v"
        d = ulp_diff(kd, k_all)
        assert (d == 0).all(), f"{what}: seq {i} k differs in {(d != 0).sum()} elements"
        q_raw, k_raw, _ = orc.split_qkv(qkv[i, :c])
        cos, sin = orc.rope_cos_sin(list(range(p, p + c)))
        q_ref, _ = orc.norm_rope_qk(q_raw, k_raw, w["q_gamma"], w["k_gamma"], cos, sin)
        assert torch.equal(q_out[i, :c].cpu(), q_ref), f"{what}: seq {i} q"


@pytest.mark.parametrize("tokens", [2, 3, 4])
def test_tokens_across_block_boundaries(cuda, tokens):
    past = [0, 1, 61, 62, 63, 64, 126, 127, 200, 1000]
    w, cache, hist, qkv, out, q_out, _ = _run(cuda, past, tokens)
    _check(w, cache, hist, qkv, out, q_out, past, [tokens] * len(past), f"T={tokens}")


@pytest.mark.parametrize("bps", [1, 2, 5])
def test_tokens_split_keys_merged_in_kernel(cuda, bps):
    """Several items per sequence (splits), merged by the kernel's merger warp."""
    past = [500, 70, 250, 900, 3]
    tokens = 4
    w, cache, hist, qkv, out, q_out, splits = _run(cuda, past, tokens, bps=bps, capacity=1000)
    assert splits > 1
    _check(w, cache, hist, qkv, out, q_out, past, [tokens] * len(past), f"bps {bps}")


def test_tokens_ragged_chunks(cuda):
    """chunk_lens: 1..4 valid tokens per sequence; the rows past a chunk are
    ignored (their contexts stay unwritten)."""
    past = [10, 63, 64, 300, 127, 0]
    chunk = [1, 4, 2, 3, 4, 1]
    w, cache, hist, qkv, out, q_out, _ = _run(cuda, past, 4, chunk=chunk)
    _check(w, cache, hist, qkv, out, q_out, past, chunk, "ragged")
    for i, c in enumerate(chunk):
        assert (out[i, c:] == 7.0).all(), f"seq {i}: rows past the chunk were written"


def test_tokens_match_the_prefill_kernel(cuda):
    """The same chunks through the tcgen05 prefill path: contexts within the
    attention tolerance of each other, and the same appended k/v."""
    past = [64, 300, 5, 1023]
    tokens = 4
    w, cache, hist, qkv, out, _, _ = _run(cuda, past, tokens, seed=3, max_ctas=7)
    attn = load_pkg("attention")
    rope = load_pkg("rope")
    cache2, _ = build_batch(past, cuda, seed=43, capacity=max(past) + tokens + 1)
    cos, sin = rope.rope_table(2048, device=cuda)
    kp, vp = cache2.pool(0)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out2 = attn.prefill(qkv.to(cuda), torch.tensor(past, dtype=torch.int32, device=cuda), k_pool=kp, v_pool=vp,
                        block_tables=cache2.block_tables(), gamma_q=w["q_gamma"].to(cuda),
                        gamma_k=w["k_gamma"].to(cuda), cos=cos, sin=sin, dev_err=err, kernel="tcgen05")
    torch.cuda.synchronize()
    assert err.item() == 0
    check_close(out, out2, "decode step tokens vs prefill kernel")
    for i, p in enumerate(past):
        ka, va = cache.read_dense(0, i, p + tokens)
        kb, vb = cache2.read_dense(0, i, p + tokens)
        assert torch.equal(ka, kb) and torch.equal(va, vb)


def test_tokens_refusals(cuda):
    attn, lib = load_pkg("attention"), load_pkg("_lib")
    past = [1000]
    cache, _ = build_batch(past, cuda, seed=1, capacity=1100)
    kp, vp = cache.pool(0)
    counters = torch.zeros(10, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.empty(1, 4, 16, 64, dtype=torch.bfloat16, device=cuda)
    args = dict(k_pool=kp, v_pool=vp, block_tables=cache.block_tables(), out=out, counters=counters, dev_err=err,
                mode=lib.B2_STORE_KV)
    qkv = rand_qkv(4, 1).reshape(1, 4, -1).to(cuda)
    with pytest.raises(lib.B2Error):          # 18 blocks at 1 per split: 18 splits > 16
        attn.decode_step_tokens(qkv, torch.tensor(past, dtype=torch.int32, device=cuda), blocks_per_split=1,
                                **args)
    with pytest.raises(ValueError):           # 5 tokens
        attn.decode_step_tokens(rand_qkv(5, 1).reshape(1, 5, -1).to(cuda),
                                torch.tensor(past, dtype=torch.int32, device=cuda), **dict(args, out=torch.empty(
                                    1, 5, 16, 64, dtype=torch.bfloat16, device=cuda)))
    torch.cuda.synchronize()
    assert err.item() == 0


def test_prefill_routes_short_chunks_to_the_step(cuda):
    """attention.prefill picks the fused step for T <= 4 (kernel="auto"): the
    same results as the reference path."""
    attn = load_pkg("attention")
    rope = load_pkg("rope")
    past = [0, 63, 129]
    tokens = 3
    w = orc.attention_weights(0)
    cache, hist = build_batch(past, cuda, seed=44, capacity=max(past) + tokens + 1)
    qkv = torch.stack([rand_qkv(tokens, 930 + i) for i in range(len(past))])
    cos, sin = rope.rope_table(512, device=cuda)
    kp, vp = cache.pool(0)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    q_out = torch.empty(len(past), tokens, 16, 64, dtype=torch.bfloat16, device=cuda)
    out = attn.prefill(qkv.to(cuda), torch.tensor(past, dtype=torch.int32, device=cuda), k_pool=kp, v_pool=vp,
                       block_tables=cache.block_tables(), gamma_q=w["q_gamma"].to(cuda),
                       gamma_k=w["k_gamma"].to(cuda), cos=cos, sin=sin, dev_err=err, q_out=q_out)
    torch.cuda.synchronize()
    assert err.item() == 0
    _check(w, cache, hist, qkv, out, q_out, past, [tokens] * len(past), "prefill auto")
