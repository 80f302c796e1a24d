"""The fused decode step against the golden fixtures that transformers itself
produced (tests/golden/lfm2_attn_L*.npz: Lfm2Attention + DynamicCache in
BF16 at cached lengths 0 ... 1000, experiments/006_lfm25_baseline.py:115-127):
the context of the new token, the appended k/v, and (config C1) the whole
attention layer — q/k/v projections, the fused step, the output projection."""
import pathlib

import numpy as np
import pytest
import torch

from conftest import load_pkg
from oracle import lfm2_attention as orc
from test_kernels_gpu import build_batch, check_close, ulp_diff

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
CASES = sorted(GOLDEN.glob("lfm2_attn_L*.npz"), key=lambda p: int(p.stem.split("L")[-1]))


@pytest.mark.parametrize("path", CASES, ids=lambda p: p.stem)
def test_fused_step_matches_hf_golden(cuda, path):
    f = dict(np.load(path))
    n = int(f["length"])
    w = orc.attention_weights(int(f["weight_seed"]))
    k, v = orc.past_cache(1000 + n, n)
    cache, _ = build_batch([n], cuda, seed=0, capacity=n + 1)
    if n:
        cache.write_dense(0, 0, k[0], v[0])
    qkv = torch.cat([orc.from_bits(f["q_raw"]), orc.from_bits(f["k_raw"]), orc.from_bits(f["v_raw"])])[None]
    runner = load_pkg("attention").PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], 1, n + 2)
    past = torch.tensor([n], dtype=torch.int32, device=cuda)
    ctx = runner.step(0, qkv.to(cuda), past, past + 1, cache.block_tables())
    torch.cuda.synchronize()
    runner.check()
    check_close(ctx[0], orc.from_bits(f["context_sdpa"]).reshape(16, 64), f"{path.stem} context")
    kd, vd = cache.read_dense(0, 0, n + 1)
    assert np.array_equal(orc.bits(vd[:, n].cpu()), f["v_appended"]), "appended v"
    d = ulp_diff(kd[:, n], orc.from_bits(f["k_appended"]))
    assert (d == 0).all(), f"appended k: {(d != 0).sum()} elements differ (max {d.max()} ulps)"


@pytest.mark.parametrize("path", [p for p in CASES if int(p.stem.split("L")[-1]) in (0, 512, 1000)],
                         ids=lambda p: p.stem)
def test_attention_layer_matches_hf_golden(cuda, path):
    """Config C1: x -> q/k/v projections (cuBLAS) -> fused step -> out_proj,
    against Lfm2Attention.forward's output (max-abs 2e-2 / relative 1e-2)."""
    f = dict(np.load(path))
    n = int(f["length"])
    w = orc.attention_weights(int(f["weight_seed"]))
    k, v = orc.past_cache(1000 + n, n)
    cache, _ = build_batch([n], cuda, seed=0, capacity=n + 1)
    if n:
        cache.write_dense(0, 0, k[0], v[0])
    x = orc.from_bits(f["x"]).reshape(1, 1024).to(cuda)
    wqkv = torch.cat([w["q_proj"], w["k_proj"], w["v_proj"]]).to(cuda)
    qkv = x @ wqkv.t()
    runner = load_pkg("attention").PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], 1, n + 2)
    past = torch.tensor([n], dtype=torch.int32, device=cuda)
    ctx = runner.step(0, qkv, past, past + 1, cache.block_tables())
    out = ctx.reshape(1, 1024) @ w["out_proj"].to(cuda).t()
    torch.cuda.synchronize()
    runner.check()
    check_close(out[0], orc.from_bits(f["output_sdpa"]).reshape(1024), f"{path.stem} layer output")
