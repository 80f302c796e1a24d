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
