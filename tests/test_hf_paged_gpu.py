"""transformers' Lfm2ForCausalLM decoding on the paged B200 path through the
Hugging Face adapter (attention implementation "b200_paged" + B200PagedCache),
with the model code unchanged.

Checked three ways:
  * teacher-forced against the reference's CPU greedy loop (transformers in
    BF16, one token per forward, experiments/010_cpu_greedy.py:43-63; fixture
    tests/golden/lfm2_greedy.npz), with the runner test's near-tie rule;
  * against the same model on the GPU with transformers' own sdpa attention and
    DynamicCache (logits within tolerance, per step);
  * a whole prompt in one forward (the tcgen05 prefill kernels) followed by
    decode steps, against the token-by-token path.
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
BF16 = torch.bfloat16


def _model(f, device, impl):
    from transformers import Lfm2Config, Lfm2ForCausalLM
    hf = load_pkg("hf_paged")
    hf.register()
    cfg = Lfm2Config(hidden_size=1024, intermediate_size=3840, num_hidden_layers=14, num_attention_heads=16,
                     num_key_value_heads=8, vocab_size=65536, norm_eps=1e-5,
                     layer_types=list(orc.LFM25_LAYER_TYPES),
                     rope_parameters={"rope_type": "default", "rope_theta": 1.0e6}, tie_word_embeddings=True)
    cfg._attn_implementation = impl
    sd = orc.lfm2_model_weights(int(f["weight_seed"]))
    h = hashlib.sha256()
    for k in sorted(sd):
        if k != "lm_head.weight":
            h.update(orc.bits(sd[k]).tobytes())
    assert h.hexdigest() == str(f["model_weights_sha256"])
    model = Lfm2ForCausalLM(cfg).to(BF16).eval()
    model.load_state_dict(sd, strict=True)
    model.tie_weights()
    return model.to(device), hf


def test_hf_model_teacher_forced_matches_reference(cuda):
    f = dict(np.load(GOLDEN))
    model, hf = _model(f, cuda, "b200_paged")
    inputs, top_v, top_i = f["inputs"], f["top_values"], f["top_indices"]
    b, steps = inputs.shape
    cache = hf.B200PagedCache(model.config, max_batch_size=b, max_cache_len=64, device=cuda, shuffle_seed=3)
    exact, worst = 0, 0.0
    with torch.no_grad():
        for t in range(steps):
            ids = torch.from_numpy(inputs[:, t:t + 1]).to(cuda)
            logits = model(ids, past_key_values=cache, use_cache=True).logits[:, -1].float().cpu().numpy()
            nxt = logits.argmax(-1)
            for s in range(b):
                ref_ids, ref_vals = top_i[s, t], top_v[s, t]
                worst = max(worst, float(np.abs(logits[s, ref_ids] - ref_vals).max()))
                if nxt[s] == ref_ids[0]:
                    exact += 1
                    continue
                ulp = 2.0 ** (np.floor(np.log2(abs(ref_vals[0]))) - 7)
                near = ref_ids[ref_vals >= ref_vals[0] - 2 * ulp]
                assert nxt[s] in near, f"step {t} seq {s}: got {nxt[s]}, reference top {ref_ids[:3]}"
    cache.check()
    assert cache.get_seq_length() == steps
    assert worst <= 0.0625, f"logits differ by {worst} at the reference's top-8"
    assert exact >= 0.8 * b * steps


def _close(a: torch.Tensor, b: torch.Tensor, what: str) -> None:
    """Logits agree within 2 bf16 ulps of their largest magnitude (the GEMMs
    around attention round to bf16 on both sides)."""
    ulp = 2.0 ** (np.floor(np.log2(b.abs().max().item())) - 7)
    err = (a - b).abs().max().item()
    assert err <= max(0.0625, 2 * ulp), f"{what}: logits differ by {err} (ulp {ulp})"


def test_hf_model_matches_sdpa_on_gpu_and_prefill(cuda):
    """Same weights and GEMMs on the GPU: b200_paged against transformers' sdpa
    + DynamicCache, token by token, and with the prompt in one forward (the
    prefill kernels) followed by decode steps."""
    from transformers.cache_utils import DynamicCache
    f = dict(np.load(GOLDEN))
    model, hf = _model(f, cuda, "b200_paged")
    ids = torch.from_numpy(f["inputs"]).to(cuda)          # [2, 23]
    b, steps = ids.shape
    prompt = 8

    def run(impl, whole_prompt):
        model.config._attn_implementation = impl
        if impl == "sdpa":
            cache = DynamicCache(config=model.config)
        else:
            cache = hf.B200PagedCache(model.config, max_batch_size=b, max_cache_len=64, device=cuda)
        out = []
        t0 = 0
        if whole_prompt:
            out += list(model(ids[:, :prompt], past_key_values=cache, use_cache=True).logits.float().unbind(1))
            t0 = prompt
        for t in range(t0, steps):
            out.append(model(ids[:, t:t + 1], past_key_values=cache, use_cache=True).logits[:, -1].float())
        if impl != "sdpa":
            cache.check()
        model.config._attn_implementation = "b200_paged"
        return out

    with torch.no_grad():
        for whole in (False, True):
            ours, ref = run("b200_paged", whole), run("sdpa", whole)
            for t in range(steps):
                _close(ours[t], ref[t], f"{'prompt in one forward' if whole else 'token by token'}, position {t}")
        # generate() drives the same cache
        first = run("b200_paged", True)[prompt - 1]
        gc = hf.B200PagedCache(model.config, max_batch_size=b, max_cache_len=64, device=cuda)
        out = model.generate(ids[:, :prompt], past_key_values=gc, max_new_tokens=4, do_sample=False)
        assert out.shape == (b, prompt + 4)
        gc.check()
        top2 = first.topk(2, dim=-1).values
        for s in range(b):
            if (top2[s, 0] - top2[s, 1]).item() > 0.125:   # a clear winner must be the one generated
                assert out[s, prompt].item() == first[s].argmax().item()


def test_hf_model_without_paged_cache_fails_loudly(cuda):
    f = dict(np.load(GOLDEN))
    model, hf = _model(f, cuda, "b200_paged")
    ids = torch.from_numpy(f["inputs"][:, :2]).to(cuda)
    with torch.no_grad(), pytest.raises(ValueError, match="B200PagedCache"):
        model(ids, use_cache=False)
