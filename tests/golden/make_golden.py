"""Generate the golden fixtures in this folder from the reference's CPU path.

The reference computes LFM2.5 attention on the CPU with Hugging Face
transformers' Lfm2Attention + DynamicCache in BF16
(experiments/006_lfm25_baseline.py:115-127, experiments/010_cpu_greedy.py:43-63).
This script runs that code itself (transformers, imported here; it is a
third-party package, not part of the reference tree) on seeded random-init
inputs and stores its outputs as uint16 bf16 bit patterns.  The real
checkpoint and the reference's own .npz fixtures (cache/*.npz) are not
available, so the inputs are the seeded generators of oracle/lfm2_attention.py;
a sha256 of every regenerated input is stored to pin the generators.

Run from the repository root:  python tests/golden/make_golden.py
(`--only greedy` / `--only greedy_free` regenerates only that greedy fixture).
Nothing at test time imports transformers; tests read the .npz files.
"""
from __future__ import annotations

import hashlib
import pathlib
import sys

import numpy as np
import torch

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import transformers  # noqa: E402
from transformers import Lfm2Config  # noqa: E402
from transformers.cache_utils import DynamicCache  # noqa: E402
from transformers.models.lfm2 import modeling_lfm2 as hf  # noqa: E402

from oracle import lfm2_attention as orc  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent
BF16 = torch.bfloat16
LAYER_TYPES = ["conv", "conv", "full_attention", "conv", "full_attention", "conv",
               "full_attention", "conv", "full_attention", "conv", "full_attention", "conv",
               "full_attention", "conv"]  # experiments/lfm25_x8.py:55-57
CASES = [0, 1, 21, 63, 64, 65, 512, 1000]   # cached tokens before the step
ROPE_POSITIONS = [0, 1, 2, 21, 63, 64, 511, 512, 1000, 4095, 8191, 16383, 65535,
                  131071, 131072, 131136]
WEIGHT_SEED = 0


def config(impl: str) -> Lfm2Config:
    cfg = Lfm2Config(hidden_size=1024, intermediate_size=3840, num_hidden_layers=14,
                     num_attention_heads=16, num_key_value_heads=8, vocab_size=65536,
                     norm_eps=1e-5, layer_types=LAYER_TYPES,
                     rope_parameters={"rope_type": "default", "rope_theta": 1.0e6})
    cfg._attn_implementation = impl
    return cfg


def sha(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(orc.bits(t).tobytes())
    return h.hexdigest()


def run_case(length: int, impl: str, weights: dict) -> dict:
    cfg = config(impl)
    attn = hf.Lfm2Attention(cfg, layer_idx=2).to(BF16).eval()
    with torch.no_grad():
        attn.q_proj.weight.copy_(weights["q_proj"])
        attn.k_proj.weight.copy_(weights["k_proj"])
        attn.v_proj.weight.copy_(weights["v_proj"])
        attn.out_proj.weight.copy_(weights["out_proj"])
        attn.q_layernorm.weight.copy_(weights["q_gamma"])
        attn.k_layernorm.weight.copy_(weights["k_gamma"])
    rotary = hf.Lfm2RotaryEmbedding(cfg)
    k_past, v_past = orc.past_cache(1000 + length, length)
    x = orc.hidden_input(2000 + length)
    cache = DynamicCache()
    if length:
        cache.update(k_past, v_past, 2)
    else:
        cache.update(k_past[:, :, :0], v_past[:, :, :0], 2)
    seen = {}
    hooks = [
        attn.q_proj.register_forward_hook(lambda m, i, o: seen.__setitem__("q_raw", o)),
        attn.k_proj.register_forward_hook(lambda m, i, o: seen.__setitem__("k_raw", o)),
        attn.v_proj.register_forward_hook(lambda m, i, o: seen.__setitem__("v_raw", o)),
        attn.q_layernorm.register_forward_hook(lambda m, i, o: seen.__setitem__("q_norm", o)),
        attn.k_layernorm.register_forward_hook(lambda m, i, o: seen.__setitem__("k_norm", o)),
        attn.out_proj.register_forward_hook(lambda m, i, o: seen.__setitem__("context", i[0])),
    ]
    with torch.no_grad():
        pos = torch.tensor([[length]])
        cos, sin = rotary(x, pos)
        out, _ = attn(x, (cos, sin), None, past_key_values=cache)
        q_rot, k_rot = hf.apply_rotary_pos_emb(seen["q_norm"].transpose(1, 2),
                                               seen["k_norm"].transpose(1, 2), cos, sin)
    for h in hooks:
        h.remove()
    layer = cache.layers[2]
    return {
        "x": orc.bits(x.reshape(-1)),
        "q_raw": orc.bits(seen["q_raw"].reshape(-1)),
        "k_raw": orc.bits(seen["k_raw"].reshape(-1)),
        "v_raw": orc.bits(seen["v_raw"].reshape(-1)),
        "q_norm": orc.bits(seen["q_norm"].reshape(16, 64)),
        "k_norm": orc.bits(seen["k_norm"].reshape(8, 64)),
        "cos": orc.bits(cos.reshape(64)),
        "sin": orc.bits(sin.reshape(64)),
        "q_rot": orc.bits(q_rot.reshape(16, 64)),
        "k_rot": orc.bits(k_rot.reshape(8, 64)),
        "k_appended": orc.bits(layer.keys[0, :, length]),
        "v_appended": orc.bits(layer.values[0, :, length]),
        "cache_len": np.int64(layer.keys.shape[2]),
        "context": orc.bits(seen["context"].reshape(16, 64)),
        "output": orc.bits(out.reshape(-1)),
        "past_sha256": sha(k_past, v_past),
        "x_sha256": sha(x),
    }


PREFILL_CASES = [(21, 5), (0, 70), (100, 64)]   # (cached tokens, chunk tokens)


def prefill_case(past: int, t: int, weights: dict) -> dict:
    """Lfm2Attention.forward on a chunk of t tokens after `past` cached ones,
    with the causal mask of a cached prefix (query i sees keys 0..past+i, the
    mask transformers' create_causal_mask builds); sdpa."""
    cfg = config("sdpa")
    attn = hf.Lfm2Attention(cfg, layer_idx=2).to(BF16).eval()
    with torch.no_grad():
        for name in ("q_proj", "k_proj", "v_proj", "out_proj"):
            getattr(attn, name).weight.copy_(weights[name])
        attn.q_layernorm.weight.copy_(weights["q_gamma"])
        attn.k_layernorm.weight.copy_(weights["k_gamma"])
    rotary = hf.Lfm2RotaryEmbedding(cfg)
    k_past, v_past = orc.past_cache(3000 + past, past)
    g = torch.Generator().manual_seed(4000 + t)
    x = torch.randn(1, t, 1024, generator=g).to(BF16)
    cache = DynamicCache()
    cache.update(k_past, v_past, 2)
    seen = {}
    hooks = [attn.out_proj.register_forward_hook(lambda m, i, o: seen.__setitem__("context", i[0])),
             attn.q_proj.register_forward_hook(lambda m, i, o: seen.__setitem__("q_raw", o)),
             attn.k_proj.register_forward_hook(lambda m, i, o: seen.__setitem__("k_raw", o)),
             attn.v_proj.register_forward_hook(lambda m, i, o: seen.__setitem__("v_raw", o))]
    keys = torch.arange(past + t)
    mask = (keys[None, :] <= (past + torch.arange(t))[:, None])[None, None]
    with torch.no_grad():
        cos, sin = rotary(x, torch.arange(past, past + t)[None])
        attn(x, (cos, sin), mask, past_key_values=cache)
    for h in hooks:
        h.remove()
    qkv = torch.cat([seen["q_raw"], seen["k_raw"], seen["v_raw"]], dim=-1)[0]
    return {"qkv": orc.bits(qkv), "context": orc.bits(seen["context"].reshape(t, 16, 64)),
            "past": np.int64(past), "tokens": np.int64(t), "past_sha256": sha(k_past, v_past)}


GREEDY_SEED = 5
GREEDY_BATCH, GREEDY_PROMPT, GREEDY_NEW, GREEDY_TOPK = 2, 8, 16, 8


def greedy_case() -> dict:
    """The reference's CPU greedy loop (experiments/010_cpu_greedy.py:43-63):
    Lfm2ForCausalLM in BF16, one token per forward with a DynamicCache, argmax.
    Records, for every step, the input ids and the top-8 logits (values and
    indices) so that a GPU runner can be checked teacher-forced.  The same
    inputs are also run with transformers' eager attention (the reference's
    other CPU attention path) and its logits at those top-8 ids recorded, to
    show how far the reference's own implementations differ."""
    from transformers import Lfm2ForCausalLM
    sd = orc.lfm2_model_weights(GREEDY_SEED)

    def model_for(impl):
        cfg = config(impl)
        cfg.tie_word_embeddings = True
        model = Lfm2ForCausalLM(cfg).to(BF16).eval()
        model.load_state_dict(sd, strict=True)
        model.tie_weights()
        return model, cfg

    model, cfg = model_for("sdpa")
    g = torch.Generator().manual_seed(GREEDY_SEED + 1)
    prompt = torch.randint(0, cfg.vocab_size, (GREEDY_BATCH, GREEDY_PROMPT), generator=g)
    cache = DynamicCache(config=cfg)
    inputs, topv, topi = [], [], []
    nxt = None
    with torch.no_grad():
        for t in range(GREEDY_PROMPT + GREEDY_NEW - 1):
            ids = prompt[:, t] if t < GREEDY_PROMPT else nxt
            logits = model(ids[:, None], past_key_values=cache, use_cache=True).logits[:, -1]
            v, i = logits.float().topk(GREEDY_TOPK, dim=-1)
            inputs.append(ids.clone())
            topv.append(v)
            topi.append(i)
            nxt = logits.argmax(-1)
    inputs, topi = torch.stack(inputs, 1), torch.stack(topi, 1)
    eager, ecfg = model_for("eager")
    cache = DynamicCache(config=ecfg)
    eager_v = []
    with torch.no_grad():
        for t in range(inputs.shape[1]):
            logits = eager(inputs[:, t:t + 1], past_key_values=cache, use_cache=True).logits[:, -1].float()
            eager_v.append(torch.gather(logits, 1, topi[:, t]))
    return {"inputs": inputs.numpy(), "top_values": torch.stack(topv, 1).numpy(),
            "top_indices": topi.numpy(), "eager_top_values": torch.stack(eager_v, 1).numpy(),
            "prompt_len": np.int64(GREEDY_PROMPT), "weight_seed": np.int64(GREEDY_SEED),
            "model_weights_sha256": sha(*[sd[k] for k in sorted(sd) if k != "lm_head.weight"])}


FREE_SEED = 7
FREE_PROMPTS, FREE_PROMPT_LEN, FREE_NEW, FREE_TOPK = 16, 32, 64, 4
EOS_ID = 7   # experiments/010_cpu_greedy.py:19


def greedy_free_case() -> dict:
    """Free-running greedy generation with the reference's CPU loop, prompt by
    prompt exactly as experiments/010_cpu_greedy.py:46-63 runs it (batch 1,
    the prompt fed one token per forward with a DynamicCache, then argmax fed
    back until FREE_NEW tokens or EOS): the C5 model shape (random init,
    seeded), 16 prompts of 32 random ids, 64 new tokens each.  Records the
    generated ids and, at every generated step, the top-FREE_TOPK logits
    (the bf16 values as float32, and their ids), so a divergence can be
    judged against the reference's own top-2 margin at that step."""
    from transformers import Lfm2ForCausalLM
    cfg = config("sdpa")
    cfg.tie_word_embeddings = True
    model = Lfm2ForCausalLM(cfg).to(BF16).eval()
    sd = orc.lfm2_model_weights(FREE_SEED)
    model.load_state_dict(sd, strict=True)
    model.tie_weights()
    g = torch.Generator().manual_seed(FREE_SEED + 1)
    prompts = torch.randint(0, cfg.vocab_size, (FREE_PROMPTS, FREE_PROMPT_LEN), generator=g)
    gen = np.full((FREE_PROMPTS, FREE_NEW), -1, dtype=np.int64)
    topv = np.zeros((FREE_PROMPTS, FREE_NEW, FREE_TOPK), dtype=np.float32)
    topi = np.zeros((FREE_PROMPTS, FREE_NEW, FREE_TOPK), dtype=np.int64)
    with torch.inference_mode():
        for s in range(FREE_PROMPTS):
            past = DynamicCache(config=cfg)
            for token in prompts[s].tolist():
                out = model(torch.tensor([[token]]), past_key_values=past, use_cache=True)
            for t in range(FREE_NEW):
                logits = out.logits[0, -1]
                v, i = logits.float().topk(FREE_TOPK)
                topv[s, t], topi[s, t] = v.numpy(), i.numpy()
                nxt = int(logits.argmax())
                gen[s, t] = nxt
                if nxt == EOS_ID or t == FREE_NEW - 1:
                    break
                out = model(torch.tensor([[nxt]]), past_key_values=past, use_cache=True)
    return {"prompts": prompts.numpy(), "generated": gen, "top_values": topv, "top_indices": topi,
            "weight_seed": np.int64(FREE_SEED), "eos_id": np.int64(EOS_ID),
            "model_weights_sha256": sha(*[sd[k] for k in sorted(sd) if k != "lm_head.weight"])}


def main() -> None:
    torch.manual_seed(0)
    if sys.argv[1:] == ["--only", "greedy"]:
        weights = orc.attention_weights(WEIGHT_SEED)
        meta = {"transformers": transformers.__version__, "torch": torch.__version__,
                "weights_sha256": sha(*[weights[k] for k in sorted(weights)])}
        np.savez_compressed(OUT / "lfm2_greedy.npz", **greedy_case(), **meta)
        print("wrote lfm2_greedy.npz")
        return
    if sys.argv[1:] == ["--only", "greedy_free"]:
        meta = {"transformers": transformers.__version__, "torch": torch.__version__}
        np.savez_compressed(OUT / "lfm2_greedy_free.npz", **greedy_free_case(), **meta)
        print("wrote lfm2_greedy_free.npz")
        return
    weights = orc.attention_weights(WEIGHT_SEED)
    meta = {"transformers": transformers.__version__, "torch": torch.__version__,
            "weights_sha256": sha(*[weights[k] for k in sorted(weights)])}
    for length in CASES:
        rec = {}
        for impl in ("sdpa", "eager"):
            r = run_case(length, impl, weights)
            for k, v in r.items():
                if impl == "sdpa" or k in ("context", "output"):
                    rec[f"{k}_{impl}" if k in ("context", "output") else k] = v
        np.savez_compressed(OUT / f"lfm2_attn_L{length}.npz", **rec, **meta, length=np.int64(length),
                            weight_seed=np.int64(WEIGHT_SEED))
    cfg = config("sdpa")
    rotary = hf.Lfm2RotaryEmbedding(cfg)
    with torch.no_grad():
        pos = torch.tensor([ROPE_POSITIONS])
        cos, sin = rotary(torch.zeros(1, dtype=BF16), pos)
    np.savez_compressed(OUT / "lfm2_rope.npz", positions=np.array(ROPE_POSITIONS, dtype=np.int64),
                        cos=orc.bits(cos[0]), sin=orc.bits(sin[0]), **meta)
    for past, t in PREFILL_CASES:
        np.savez_compressed(OUT / f"lfm2_prefill_P{past}_T{t}.npz", **prefill_case(past, t, weights), **meta,
                            weight_seed=np.int64(WEIGHT_SEED))
    np.savez_compressed(OUT / "lfm2_greedy.npz", **greedy_case(), **meta)
    np.savez_compressed(OUT / "lfm2_greedy_free.npz", **greedy_free_case(),
                        **{k: meta[k] for k in ("transformers", "torch")})
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    main()
