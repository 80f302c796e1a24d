"""Whole-model decode (config C5 shape) through the paged attention path,
against the reference's CPU greedy loop (transformers Lfm2ForCausalLM in
BF16, one token per forward: experiments/010_cpu_greedy.py:43-63).

The reference's own criterion compares the generated id sequences token for
token (experiments/010_compare.py:33-51) and explains a divergence by the CPU
logits at that step: an exact bf16 top-2 tie, or top-2 logits one bf16 step
apart (experiments/010_x8_engine.md:59-69).  Logits are not bit-exact across
implementations: the reference's own two CPU attention paths (sdpa and
eager) differ by up to 2 bf16 ulps at the top candidates
(tests/test_oracle.py::test_reference_cpu_paths_differ_by_a_few_ulps), and
the GPU's GEMMs and split softmax (fp32, other orders) land within 3 ulps of
the sdpa path.  So every logit at the reference's top-8 must be within
TIE_ULPS = 3 ulps of the reference's, and every greedy choice must equal the
reference's except where two of the reference's top candidates lie close
enough for those errors to swap them: within 2 * TIE_ULPS ulps (one logit up
to TIE_ULPS high, the other up to TIE_ULPS low); the choice must then be one
of those candidates.
"""
import hashlib
import pathlib

import numpy as np
import pytest
import torch

from conftest import load_pkg
from oracle import lfm2_attention as orc

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "lfm2_greedy.npz"
FREE = pathlib.Path(__file__).resolve().parent / "golden" / "lfm2_greedy_free.npz"


TIE_ULPS = 3


def bf16_ulp(x: float) -> float:
    return 2.0 ** (np.floor(np.log2(abs(x))) - 7)


def _weights(f):
    sd = orc.lfm2_model_weights(int(f["weight_seed"]))
    h = hashlib.sha256()
    for k in sorted(sd):
        if k != "lm_head.weight":
            h.update(orc.bits(sd[k]).tobytes())
    assert h.hexdigest() == str(f["model_weights_sha256"])
    return sd


@pytest.mark.parametrize("glue", ["kernels", "kernels_cublas", "torch_glue"])
@pytest.mark.parametrize("use_graph", [True, False], ids=["graph", "eager"])
def test_greedy_teacher_forced_matches_reference(cuda, use_graph, glue):
    """Teacher-forced (the reference's inputs at every step): the logits at the
    reference's top-8 within TIE_ULPS bf16 ulps of the reference's; the argmax
    equals the reference's except where its top logits are within 2 * TIE_ULPS
    ulps of each other, and then it is one of those (any of the top-8)."""
    f = dict(np.load(GOLDEN))
    runner_mod = load_pkg("lfm2_runner")
    inputs = f["inputs"]                      # [B, T]
    top_v, top_i = f["top_values"], f["top_indices"]
    b, steps = inputs.shape
    runner = runner_mod.LFM2DecodeRunner(_weights(f), max_batch=b, max_context=64, device=cuda,
                                         use_graph=use_graph, fused_glue=glue != "torch_glue",
                                         own_gemm=glue == "kernels")
    ulps, flips = [], []
    for t in range(steps):
        nxt = runner.step(torch.from_numpy(inputs[:, t])).cpu().numpy()
        logits = runner.logits.float().cpu().numpy()
        for s in range(b):
            ref_ids, ref_vals = top_i[s, t], top_v[s, t]
            ulps.extend(np.abs(logits[s, ref_ids] - ref_vals) / np.array([bf16_ulp(v) for v in ref_vals]))
            if nxt[s] != ref_ids[0]:
                flips.append((t, s, int(nxt[s]), ref_ids.tolist(), ref_vals.tolist()))
    runner.check()
    hist = np.bincount(np.minimum(np.round(ulps).astype(int), 8))
    print(f"logit differences at the reference's top-8, in bf16 ulps (0..8+): {hist.tolist()}; flips {flips}")
    assert len(hist) <= TIE_ULPS + 1, f"logits beyond {TIE_ULPS} ulps of the reference: {hist.tolist()}"
    for t, s, got, ids, vals in flips:
        # candidates: the reference's top-8 within 2 * TIE_ULPS of its top logit
        near = [i for i, v in zip(ids, vals) if v >= vals[0] - 2 * TIE_ULPS * bf16_ulp(vals[0])]
        assert got in near, f"step {t} seq {s}: got {got}, reference top {ids[:4]} {vals[:4]}"
    k, v = runner.kv(0, 0, steps - 1)
    assert k.shape == (8, steps, 64) and torch.isfinite(k.float()).all() and torch.isfinite(v.float()).all()


@pytest.mark.parametrize("own_gemm", [True, False], ids=["b2_gemm", "cublas"])
def test_greedy_free_running_matches_reference(cuda, own_gemm):
    """Free-running greedy generation, as the reference's 010_compare.py runs
    it: 16 prompts of 32 random ids (C5 model shape), 64 new tokens each, the
    GPU feeding back its own choices.  Each prompt's generated ids equal the
    reference's up to the first divergence (the comparison of that prompt ends
    there, as the two generations then continue from different tokens).  Up
    to it the histories are identical, so every logit is within TIE_ULPS of
    the reference's, as the teacher-forced test checks; two candidates can
    then change order only if the reference's logits of the two are at most
    2 * TIE_ULPS apart.  A divergence is accepted only there: the GPU's choice
    is among the reference's top-8 and within 2 * TIE_ULPS bf16 ulps of its
    top logit.  (Measured: divergences at reference gaps of 0-4 ulps with
    either GEMM, about 12 tokens into a prompt; an exact tie in 3-4 of 16.)"""
    f = dict(np.load(FREE))
    runner_mod = load_pkg("lfm2_runner")
    prompts, ref = f["prompts"], f["generated"]
    top_v, top_i = f["top_values"], f["top_indices"]
    n, new = ref.shape
    runner = runner_mod.LFM2DecodeRunner(_weights(f), max_batch=n, max_context=prompts.shape[1] + new + 1,
                                         device=cuda, own_gemm=own_gemm)
    got = runner.generate(torch.from_numpy(prompts), new).cpu().numpy()
    runner.check()
    compared, report = 0, []
    for s in range(n):
        diff = np.nonzero(got[s] != ref[s])[0]
        first = int(diff[0]) if diff.size else new
        compared += first
        if first == new:
            continue
        v, i = top_v[s, first], top_i[s, first]
        near = i[v >= v[0] - 2 * TIE_ULPS * bf16_ulp(v[0])]
        assert got[s, first] in near, \
            f"prompt {s} diverges at token {first}: got {got[s, first]}, reference top {i[:4]} {v[:4]}"
        gap = (v[0] - v[list(i).index(got[s, first])]) / bf16_ulp(v[0])
        report.append((s, first, int(got[s, first]), int(i[0]), float(gap)))
    print(f"greedy free-running: {compared} of {n * new} tokens identical before any divergence; "
          f"divergences (prompt, token, got, ref top-1, reference gap in ulps): {report}")


def test_generate_and_reset(cuda):
    runner_mod = load_pkg("lfm2_runner")
    f = dict(np.load(GOLDEN))
    runner = runner_mod.LFM2DecodeRunner(_weights(f), max_batch=2, max_context=40, device=cuda)
    prompt = torch.from_numpy(f["inputs"][:, :8])
    a = runner.generate(prompt, 6).cpu()
    runner.reset()
    b = runner.generate(prompt, 6).cpu()
    runner.check()
    assert a.shape == (2, 6) and torch.equal(a, b)
    with pytest.raises(ValueError):
        runner.step(torch.zeros(3, dtype=torch.long))


@pytest.mark.parametrize("own_gemm", [True, False], ids=["b2_gemm", "cublas"])
def test_kernel_glue_matches_torch_glue(cuda, own_gemm):
    """The same model, token by token, with the layer glue in libb2attn.so and
    as torch ops, around the same projections (b2_gemm, or cuBLAS): logits
    within a few bf16 ulps of their scale."""
    runner_mod = load_pkg("lfm2_runner")
    f = dict(np.load(GOLDEN))
    sd = _weights(f)
    ids = torch.from_numpy(f["inputs"])
    runs = []
    for fused in (True, False):
        r = runner_mod.LFM2DecodeRunner(sd, max_batch=ids.shape[0], max_context=40, device=cuda, fused_glue=fused,
                                        own_gemm=own_gemm)
        logits = []
        for t in range(12):
            r.step(ids[:, t])
            logits.append(r.logits.float().clone())
        r.check()
        runs.append(torch.stack(logits))
    scale = runs[1].abs().max().item()
    err = (runs[0] - runs[1]).abs().max().item()
    assert err <= max(0.0625, 4 * 2.0 ** (np.floor(np.log2(scale)) - 7)), f"logits differ by {err} (scale {scale})"
