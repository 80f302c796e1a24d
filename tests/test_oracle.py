"""The CPU oracle against golden vectors produced by the reference's own CPU
path (transformers Lfm2Attention + DynamicCache, see tests/golden/make_golden.py)."""
import hashlib
import pathlib

import numpy as np
import pytest
import torch

from oracle import lfm2_attention as orc

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
CASES = sorted(GOLDEN.glob("lfm2_attn_L*.npz"), key=lambda p: int(p.stem.split("L")[1]))


def _sha(*ts):
    h = hashlib.sha256()
    for t in ts:
        h.update(orc.bits(t).tobytes())
    return h.hexdigest()


def _load(path):
    return dict(np.load(path))


def test_golden_present():
    assert len(CASES) >= 8
    assert (GOLDEN / "lfm2_rope.npz").exists()


def test_generators_pinned():
    f = _load(CASES[0])
    w = orc.attention_weights(int(f["weight_seed"]))
    assert _sha(*[w[k] for k in sorted(w)]) == str(f["weights_sha256"])
    for path in CASES:
        f = _load(path)
        n = int(f["length"])
        k, v = orc.past_cache(1000 + n, n)
        assert _sha(k, v) == str(f["past_sha256"])
        assert _sha(orc.hidden_input(2000 + n)) == str(f["x_sha256"])


def test_rope_tables_match_hf():
    f = _load(GOLDEN / "lfm2_rope.npz")
    cos, sin = orc.rope_cos_sin(f["positions"])
    assert np.array_equal(orc.bits(cos), f["cos"])
    assert np.array_equal(orc.bits(sin), f["sin"])


@pytest.mark.parametrize("path", CASES, ids=lambda p: p.stem)
def test_norm_rope_bit_exact(path):
    f = _load(path)
    w = orc.attention_weights(int(f["weight_seed"]))
    q_raw = orc.from_bits(f["q_raw"]).reshape(1, 16, 64)
    k_raw = orc.from_bits(f["k_raw"]).reshape(1, 8, 64)
    qn = orc.rms_norm(q_raw, w["q_gamma"])
    kn = orc.rms_norm(k_raw, w["k_gamma"])
    assert np.array_equal(orc.bits(qn[0]), f["q_norm"])
    assert np.array_equal(orc.bits(kn[0]), f["k_norm"])
    cos, sin = orc.rope_cos_sin([int(f["length"])])
    assert np.array_equal(orc.bits(cos[0]), f["cos"])
    q, k = orc.norm_rope_qk(q_raw, k_raw, w["q_gamma"], w["k_gamma"], cos, sin)
    assert np.array_equal(orc.bits(q[0]), f["q_rot"])
    assert np.array_equal(orc.bits(k[0]), f["k_rot"])
    assert np.array_equal(f["k_appended"], f["k_rot"])


@pytest.mark.parametrize("impl", ["sdpa", "eager"])
@pytest.mark.parametrize("path", CASES, ids=lambda p: p.stem)
def test_layer_step_matches_hf(path, impl):
    f = _load(path)
    n = int(f["length"])
    w = orc.attention_weights(int(f["weight_seed"]))
    k, v = orc.past_cache(1000 + n, n)
    x = orc.hidden_input(2000 + n)
    out, ctx, qkv = orc.attention_layer_step(x, w, k[0], v[0], n, impl)
    assert np.array_equal(orc.bits(qkv[:1024]), f["q_raw"])
    assert np.array_equal(orc.bits(ctx), f[f"context_{impl}"])
    assert np.array_equal(orc.bits(out.reshape(-1)), f[f"output_{impl}"])


def test_merge_states_equals_full_attention():
    g = torch.Generator().manual_seed(5)
    q = torch.randn(16, 64, generator=g).to(orc.BF16)
    k = torch.randn(8, 300, 64, generator=g).to(orc.BF16)
    v = torch.randn(8, 300, 64, generator=g).to(orc.BF16)
    full = orc.attend(q[None, :, None, :], k[None], v[None], "fp32").reshape(16, 64)
    parts = [orc.partial_state(q, k[:, a:b], v[:, a:b]) for a, b in [(0, 64), (64, 64), (64, 250), (250, 300)]]
    assert torch.allclose(orc.merge_states(parts), full, atol=1e-5, rtol=1e-5)


def test_paged_round_trip():
    rng = np.random.default_rng(0)
    k = rng.integers(0, 65535, size=(8, 150, 64), dtype=np.uint16)
    v = rng.integers(0, 65535, size=(8, 150, 64), dtype=np.uint16)
    pool_k = np.zeros((10, 8, 64, 64), np.uint16)
    pool_v = np.zeros_like(pool_k)
    table = np.array([7, 2, 5], np.int32)
    orc.paged_from_dense(k, v, table, pool_k, pool_v)
    assert np.array_equal(orc.dense_from_paged(pool_k, table, 150), k)
    assert np.array_equal(orc.dense_from_paged(pool_v, table, 150), v)


def test_ref_layouts():
    rng = np.random.default_rng(1)
    qkv = rng.integers(0, 65535, size=3072, dtype=np.uint16)
    prior = rng.integers(0, 65535, size=8 * 2 * 21 * 64, dtype=np.uint16)
    nxt = orc.ref_append_cache(qkv, prior).reshape(8, 2, 22, 64)
    assert np.array_equal(nxt[:, :, :21].reshape(-1), prior)
    assert np.array_equal(nxt[3, 0, 21], qkv[1024 + 192:1024 + 256])
    assert np.array_equal(nxt[3, 1, 21], qkv[1536 + 192:1536 + 256])
    assert orc.float_to_bf16_bits(np.float32(22.0)) == 0x41B0


PREFILL = sorted(GOLDEN.glob("lfm2_prefill_*.npz"))


@pytest.mark.parametrize("path", PREFILL, ids=lambda p: p.stem)
def test_prefill_oracle_matches_hf(path):
    f = _load(path)
    past, t = int(f["past"]), int(f["tokens"])
    w = orc.attention_weights(int(f["weight_seed"]))
    k, v = orc.past_cache(3000 + past, past)
    assert _sha(k, v) == str(f["past_sha256"])
    ctx, k_all, v_all = orc.prefill_step(orc.from_bits(f["qkv"]).reshape(t, -1), k[0], v[0], past,
                                         w["q_gamma"], w["k_gamma"])
    assert np.array_equal(orc.bits(ctx), f["context"])
    assert k_all.shape == (8, past + t, 64)


def sum_squares64_kernel_order(x: np.ndarray) -> np.ndarray:
    """The order in which the decode and append kernels add the 64 rounded
    squares of a head vector (csrc/b2_attn.cu, sum_squares64), restated in
    numpy float32 with no fused multiply-add: v_k = squares 8k..8k+7,
    a_k = v_k + v_{k+4}, p = ((a_0 + a_1) + a_2) + a_3 lane-wise, then the 8
    lanes of p added left to right."""
    f32 = np.float32
    sq = (x.astype(f32) * x.astype(f32)).astype(f32)
    v = [sq[:, 8 * k: 8 * k + 8] for k in range(8)]
    a = [(v[k] + v[k + 4]).astype(f32) for k in range(4)]
    p = (((a[0] + a[1]).astype(f32) + a[2]).astype(f32) + a[3]).astype(f32)
    s = p[:, 0].copy()
    for lane in range(1, 8):
        s = (s + p[:, lane]).astype(f32)
    return s


@pytest.mark.parametrize("scale", [1e-3, 0.6, 1.0, 37.0])
def test_kernel_sum_order_is_torch_mean_order(scale):
    """torch's CPU x.pow(2).mean(-1) of a contiguous 64-float row (the
    variance of Lfm2RMSNorm, modeling_lfm2.py:59-64) equals the kernels'
    summation order divided by 64, bit for bit, on 100 000 bf16 rows.  This
    pins the order the append kernels reproduce for a bit-exact KV append."""
    g = torch.Generator().manual_seed(int(scale * 1000))
    x = (torch.randn(100_000, 64, generator=g) * scale).to(torch.bfloat16).float()
    ref = x.pow(2).mean(-1).numpy()
    got = sum_squares64_kernel_order(x.numpy()) / np.float32(64)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_kernel_sum_order_on_golden_heads():
    """The same on every q/k head vector of the transformers fixtures."""
    for path in CASES:
        f = _load(path)
        x = np.concatenate([orc.from_bits(f["q_raw"]).reshape(16, 64).float().numpy(),
                            orc.from_bits(f["k_raw"]).reshape(8, 64).float().numpy()])
        ref = torch.from_numpy(x).pow(2).mean(-1).numpy()
        got = sum_squares64_kernel_order(x) / np.float32(64)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), path.stem


def test_package_rope_table_matches_hf():
    """The product's RoPE table (rope.rope_table, what every kernel reads)
    against transformers' Lfm2RotaryEmbedding at the fixture's positions,
    up to 131 136 (the long-context config's range)."""
    from conftest import load_pkg
    f = _load(GOLDEN / "lfm2_rope.npz")
    pos = np.asarray(f["positions"], dtype=np.int64)
    cos, sin = load_pkg("rope").rope_table(int(pos.max()) + 1, device="cpu")
    assert np.array_equal(orc.bits(cos[pos]), f["cos"])
    assert np.array_equal(orc.bits(sin[pos]), f["sin"])


def test_reference_cpu_paths_differ_by_a_few_ulps():
    """The reference's own two CPU attention paths (transformers sdpa, which
    produced the greedy fixture, and eager) on the same teacher-forced inputs
    of the C5-shaped model: their logits at the sdpa top-8 differ by up to
    2 bf16 ulps (GEMM and softmax roundings in another order), and the
    greedy choice can differ where the top candidates are that close.  This
    is the noise floor against which the GPU runner's greedy parity is read."""
    f = _load(GOLDEN / "lfm2_greedy.npz")
    v, e = f["top_values"], f["eager_top_values"]
    ulp = 2.0 ** (np.floor(np.log2(np.abs(v))) - 7)
    d = np.round(np.abs(e - v) / ulp).astype(int)
    assert d.max() == 2 and (d > 0).mean() > 0.3
