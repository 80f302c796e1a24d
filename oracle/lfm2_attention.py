"""CPU oracle for the LFM2.5 decode-attention path.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
import this module, and only as the checker or the timed CPU baseline.  The
product (the package next to this folder) never imports it: its compute path
is libb2attn.so and has no CPU fallback.

What it restates.  The reference's CPU path for this hot path is Hugging Face
transformers' Lfm2Attention in BF16 with a DynamicCache
(006_lfm25_baseline.py:115-127, 010_cpu_greedy.py:43-63,
006_lfm25_attention_prefix_reference.py:12,56-66 import it).  transformers is a
third-party dependency, not part of the reference tree; the reference pinned
5.5.4 (docs/setup.md:31), this image has 5.5.0.  Its published algorithm,
restated below with the same torch CPU operations in the same order:

  Lfm2RMSNorm.forward            modeling_lfm2.py:59-64
  compute_default_rope_parameters / Lfm2RotaryEmbedding.forward  :93-132
  rotate_half / apply_rotary_pos_emb                            :143-185
  repeat_kv / eager_attention_forward                           :188-223
  sdpa_attention_forward (enable_gqa path)   integrations/sdpa_attention.py:40-100
  DynamicLayer.update (torch.cat along T)    cache_utils.py:102-120
  Lfm2Attention.forward                      modeling_lfm2.py:244-281

The reference's NPU operators (byte layouts of their caches and packed tail,
experiments/kernels/lfm25_attention_*.cc) are restated with numpy in
`ref_*` functions; those are pure data movement and are compared bit-exactly.

Pinning: tests/golden/make_golden.py runs the real transformers code on seeded
inputs and stores its outputs in tests/golden/*.npz; tests/test_oracle.py
checks this module against them.
"""
from __future__ import annotations

import numpy as np
import torch

BF16 = torch.bfloat16
HQ, HKV, D, BLOCK = 16, 8, 64, 64
QKV_WIDTH = (HQ + 2 * HKV) * D
THETA = 1.0e6
EPS = 1.0e-5
SCALE = D ** -0.5


# ----------------------------------------------------------------- seeded inputs

def attention_weights(seed: int, hidden: int = 1024) -> dict[str, torch.Tensor]:
    """Random-init LFM2.5 attention weights: linears N(0, 0.02) (the config's
    initializer_range), q/k RMSNorm gains 1 + N(0, 0.1) so that gamma matters."""
    g = torch.Generator().manual_seed(seed)
    w = {
        "q_proj": torch.randn(HQ * D, hidden, generator=g) * 0.02,
        "k_proj": torch.randn(HKV * D, hidden, generator=g) * 0.02,
        "v_proj": torch.randn(HKV * D, hidden, generator=g) * 0.02,
        "out_proj": torch.randn(hidden, HQ * D, generator=g) * 0.02,
        "q_gamma": 1.0 + 0.1 * torch.randn(D, generator=g),
        "k_gamma": 1.0 + 0.1 * torch.randn(D, generator=g),
    }
    return {k: v.to(BF16) for k, v in w.items()}


LFM25_LAYER_TYPES = ("conv", "conv", "full_attention", "conv", "full_attention", "conv", "full_attention",
                     "conv", "full_attention", "conv", "full_attention", "conv", "full_attention", "conv")


def lfm2_model_weights(seed: int, hidden: int = 1024, ffn: int = 2560, vocab: int = 65536,
                       layer_types=LFM25_LAYER_TYPES, conv_l: int = 3) -> dict[str, torch.Tensor]:
    """Random-init LFM2.5-230M-shaped weights with Hugging Face parameter names
    (the layer pattern of experiments/lfm25_x8.py:55-57, FFN width 2560 of
    experiments/lfm25_x8.py:50): matrices N(0, 0.02) (the config's
    initializer_range), RMSNorm gains 1, q/k layernorm gains 1 + N(0, 0.1);
    lm_head tied to the embedding.  bf16."""
    g = torch.Generator().manual_seed(seed)

    def n(*shape, std=0.02):
        return (torch.randn(*shape, generator=g) * std).to(BF16)

    sd = {"model.embed_tokens.weight": n(vocab, hidden)}
    for i, kind in enumerate(layer_types):
        p = f"model.layers.{i}."
        if kind == "full_attention":
            sd[p + "self_attn.q_proj.weight"] = n(HQ * D, hidden)
            sd[p + "self_attn.k_proj.weight"] = n(HKV * D, hidden)
            sd[p + "self_attn.v_proj.weight"] = n(HKV * D, hidden)
            sd[p + "self_attn.out_proj.weight"] = n(hidden, HQ * D)
            sd[p + "self_attn.q_layernorm.weight"] = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF16)
            sd[p + "self_attn.k_layernorm.weight"] = (1.0 + 0.1 * torch.randn(D, generator=g)).to(BF16)
        else:
            sd[p + "conv.conv.weight"] = n(hidden, 1, conv_l, std=0.3)
            sd[p + "conv.in_proj.weight"] = n(3 * hidden, hidden)
            sd[p + "conv.out_proj.weight"] = n(hidden, hidden)
        sd[p + "feed_forward.w1.weight"] = n(ffn, hidden)
        sd[p + "feed_forward.w3.weight"] = n(ffn, hidden)
        sd[p + "feed_forward.w2.weight"] = n(hidden, ffn)
        sd[p + "operator_norm.weight"] = torch.ones(hidden, dtype=BF16)
        sd[p + "ffn_norm.weight"] = torch.ones(hidden, dtype=BF16)
    sd["model.embedding_norm.weight"] = torch.ones(hidden, dtype=BF16)
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    return sd


def past_cache(seed: int, length: int, batch: int = 1) -> tuple[torch.Tensor, torch.Tensor]:
    """K, V ~ N(0, 1) in bf16, shape [batch, 8, length, 64] (DynamicCache layout)."""
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(batch, HKV, length, D, generator=g).to(BF16)
    v = torch.randn(batch, HKV, length, D, generator=g).to(BF16)
    return k, v


def hidden_input(seed: int, batch: int = 1, hidden: int = 1024) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(batch, 1, hidden, generator=g).to(BF16)


# ----------------------------------------------------------------- HF restatement

def rope_inv_freq(head_dim: int = D, theta: float = THETA) -> torch.Tensor:
    """compute_default_rope_parameters (modeling_lfm2.py:93-116)."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim))


def rope_cos_sin(positions, head_dim: int = D, theta: float = THETA) -> tuple[torch.Tensor, torch.Tensor]:
    """Lfm2RotaryEmbedding.forward (modeling_lfm2.py:118-132) for a 1-D list
    of positions: fp32 phases, cos/sin cast to bf16.  Returns [T, 64] each."""
    pos = torch.as_tensor(positions, dtype=torch.int64).reshape(1, -1)
    inv = rope_inv_freq(head_dim, theta)
    inv_expanded = inv[None, :, None].float().expand(1, -1, 1)
    freqs = (inv_expanded.float() @ pos[:, None, :].float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos = emb.cos() * 1.0
    sin = emb.sin() * 1.0
    return cos.to(BF16)[0], sin.to(BF16)[0]


def rms_norm(x: torch.Tensor, gamma: torch.Tensor, eps: float = EPS) -> torch.Tensor:
    """Lfm2RMSNorm.forward (modeling_lfm2.py:59-64)."""
    dtype = x.dtype
    h = x.to(torch.float32)
    var = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(var + eps)
    return gamma * h.to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """One operand of apply_rotary_pos_emb (modeling_lfm2.py:163-185)."""
    return (x * cos) + (rotate_half(x) * sin)


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    b, h, t, d = x.shape
    if n_rep == 1:
        return x
    return x[:, :, None, :, :].expand(b, h, n_rep, t, d).reshape(b, h * n_rep, t, d)


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, impl: str = "sdpa",
           scale: float = SCALE) -> torch.Tensor:
    """Decode attention of q [B, 16, 1, 64] over k, v [B, 8, T, 64] (bf16), no
    mask (one query attends to every cached token).  Returns [B, 1, 16, 64]
    like the attention interfaces (output transposed to [B, T, H, D])."""
    if impl == "eager":  # eager_attention_forward, modeling_lfm2.py:200-223
        ks = repeat_kv(k, HQ // HKV)
        vs = repeat_kv(v, HQ // HKV)
        w = torch.matmul(q, ks.transpose(2, 3)) * scale
        w = torch.nn.functional.softmax(w, dim=-1, dtype=torch.float32).to(q.dtype)
        out = torch.matmul(w, vs)
    elif impl == "sdpa":  # sdpa_attention_forward with enable_gqa (mask None)
        out = torch.nn.functional.scaled_dot_product_attention(
            q, k, v, attn_mask=None, dropout_p=0.0, scale=scale, is_causal=False, enable_gqa=True)
    elif impl == "fp32":  # exact-softmax fp32 reference for error budgets
        ks = repeat_kv(k.float(), HQ // HKV)
        vs = repeat_kv(v.float(), HQ // HKV)
        w = torch.softmax(torch.matmul(q.float(), ks.transpose(2, 3)) * scale, dim=-1)
        out = torch.matmul(w, vs)
    else:
        raise ValueError(impl)
    return out.transpose(1, 2).contiguous()


def split_qkv(qkv: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """[B, >=2048] -> q [B, 16, 64], k [B, 8, 64], v [B, 8, 64]."""
    b = qkv.shape[0]
    q = qkv[:, : HQ * D].reshape(b, HQ, D)
    k = qkv[:, HQ * D: (HQ + HKV) * D].reshape(b, HKV, D)
    v = qkv[:, (HQ + HKV) * D: QKV_WIDTH].reshape(b, HKV, D)
    return q, k, v


def norm_rope_qk(q_raw, k_raw, gamma_q, gamma_k, cos, sin, eps: float = EPS,
                 norm: bool = True, rope: bool = True):
    """q_layernorm/k_layernorm then apply_rotary_pos_emb for one token per
    sequence: q_raw [B, 16, 64], k_raw [B, 8, 64], cos/sin [B, 64]."""
    q, k = q_raw, k_raw
    if norm:
        q = rms_norm(q, gamma_q, eps)
        k = rms_norm(k, gamma_k, eps)
    if rope:
        c = cos[:, None, :]
        s = sin[:, None, :]
        q = apply_rope(q, c, s)
        k = apply_rope(k, c, s)
    return q, k


def decode_step(qkv_row: torch.Tensor, k_past: torch.Tensor, v_past: torch.Tensor,
                position: int, gamma_q, gamma_k, impl: str = "sdpa", eps: float = EPS,
                cos=None, sin=None):
    """One sequence, one attention layer, one token, projections excluded:
    Lfm2Attention.forward from the q/k/v projections on (modeling_lfm2.py:254-277).
    qkv_row [2048] bf16; k_past/v_past [8, L, 64].  Returns (context [16, 64],
    k_all [8, L+1, 64], v_all [8, L+1, 64], q_rot [16, 64])."""
    q_raw, k_raw, v = split_qkv(qkv_row.reshape(1, -1))
    if cos is None:
        cos, sin = rope_cos_sin([position])
    q, k = norm_rope_qk(q_raw, k_raw, gamma_q, gamma_k, cos.reshape(1, D), sin.reshape(1, D), eps)
    k_all = torch.cat([k_past.reshape(1, HKV, -1, D), k[:, :, None, :]], dim=-2)
    v_all = torch.cat([v_past.reshape(1, HKV, -1, D), v[:, :, None, :]], dim=-2)
    ctx = attend(q[:, :, None, :], k_all, v_all, impl)
    return ctx.reshape(HQ, D), k_all[0], v_all[0], q[0]


def prefill_step(qkv_rows: torch.Tensor, k_past: torch.Tensor, v_past: torch.Tensor, past: int,
                 gamma_q, gamma_k, eps: float = EPS):
    """A chunk of T new tokens of one sequence through Lfm2Attention.forward
    from the projections on (modeling_lfm2.py:254-277 with T > 1): per-token
    q/k norm + RoPE at positions past..past+T-1, the cache grown by the T
    rows, and sdpa with the causal mask transformers builds for a cached
    prefix (query t sees keys 0..past+t; with a mask, sdpa gets repeat_kv'd
    K/V, integrations/sdpa_attention.py:57-60).  qkv_rows [T, 2048];
    k_past/v_past [8, past, 64].  Returns (context [T, 16, 64], k_all, v_all)."""
    t = qkv_rows.shape[0]
    q_raw, k_raw, v = split_qkv(qkv_rows)
    cos, sin = rope_cos_sin(list(range(past, past + t)))
    q, k = norm_rope_qk(q_raw, k_raw, gamma_q, gamma_k, cos, sin, eps)    # [T, 16, 64], [T, 8, 64]
    k_all = torch.cat([k_past, k.transpose(0, 1)], dim=1)                # [8, past+T, 64]
    v_all = torch.cat([v_past, v.transpose(0, 1)], dim=1)
    keys = torch.arange(past + t)
    mask = keys[None, :] <= (past + torch.arange(t))[:, None]            # [T, past+T] bool
    out = torch.nn.functional.scaled_dot_product_attention(
        q.transpose(0, 1)[None], repeat_kv(k_all[None], HQ // HKV), repeat_kv(v_all[None], HQ // HKV),
        attn_mask=mask[None, None], dropout_p=0.0, scale=SCALE)
    return out[0].transpose(0, 1).contiguous(), k_all, v_all


def attention_layer_step(x: torch.Tensor, w: dict, k_past: torch.Tensor, v_past: torch.Tensor,
                         position: int, impl: str = "sdpa"):
    """Whole Lfm2Attention.forward for one decode token (config C1): x [1, 1, H].
    Returns (output [1, 1, H], context [16, 64], qkv_row [2048])."""
    q = torch.nn.functional.linear(x, w["q_proj"])
    k = torch.nn.functional.linear(x, w["k_proj"])
    v = torch.nn.functional.linear(x, w["v_proj"])
    qkv = torch.cat([q, k, v], dim=-1).reshape(-1)
    ctx, _, _, _ = decode_step(qkv, k_past, v_past, position, w["q_gamma"], w["k_gamma"], impl)
    out = torch.nn.functional.linear(ctx.reshape(1, 1, HQ * D), w["out_proj"])
    return out, ctx, qkv


# ----------------------------------------------------------------- partial softmax states

def partial_state(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float = SCALE):
    """fp32 (m, l, o) of q [16, 64] over k, v [8, T, 64] for a later merge;
    m in natural-log units.  T == 0 gives (-inf, 0, 0)."""
    qf = q.float().reshape(HKV, HQ // HKV, D)
    if k.shape[1] == 0:
        return (torch.full((HQ,), -float("inf")), torch.zeros(HQ), torch.zeros(HQ, D))
    s = torch.einsum("hgd,htd->hgt", qf, k.float()) * scale
    m = s.amax(-1)
    p = torch.exp(s - m[..., None])
    return m.reshape(HQ), p.sum(-1).reshape(HQ), torch.einsum("hgt,htd->hgd", p, v.float()).reshape(HQ, D)


def merge_states(states) -> torch.Tensor:
    """Log-sum-exp merge of [(m, l, o), ...] -> fp32 context [16, 64]."""
    ms = torch.stack([s[0] for s in states])
    big = ms.amax(0)
    w = torch.exp(ms - big)
    w = torch.where(torch.isfinite(ms), w, torch.zeros_like(w))
    l = (torch.stack([s[1] for s in states]) * w).sum(0)
    o = (torch.stack([s[2] for s in states]) * w[..., None]).sum(0)
    return o / l[:, None]


# ----------------------------------------------------------------- paged layout (index work)

def paged_from_dense(k: np.ndarray, v: np.ndarray, table: np.ndarray, pool_k: np.ndarray,
                     pool_v: np.ndarray) -> None:
    """Scatter dense per-sequence K/V [8, T, 64] into pool blocks
    [num_blocks, 8, 64, 64] following table (logical block -> pool block)."""
    t = k.shape[1]
    for j in range((t + BLOCK - 1) // BLOCK):
        n = min(BLOCK, t - j * BLOCK)
        pool_k[table[j], :, :n] = k[:, j * BLOCK: j * BLOCK + n]
        pool_v[table[j], :, :n] = v[:, j * BLOCK: j * BLOCK + n]


def dense_from_paged(pool: np.ndarray, table: np.ndarray, length: int) -> np.ndarray:
    """Gather [8, length, 64] from the pool (inverse of paged_from_dense)."""
    nb = (length + BLOCK - 1) // BLOCK
    if nb == 0:
        return pool[:0, :, :0].reshape(HKV, 0, D) if pool.ndim == 4 else np.zeros((HKV, 0, D), pool.dtype)
    blocks = pool[np.asarray(table[:nb])]            # [nb, 8, 64, 64]
    return blocks.transpose(1, 0, 2, 3).reshape(HKV, nb * BLOCK, D)[:, :length]


# ----------------------------------------------------------------- reference NPU operator layouts

def ref_append_cache(qkv: np.ndarray, prior: np.ndarray) -> np.ndarray:
    """lfm25_attention_append_cache_dynamic
    (experiments/kernels/lfm25_attention_append_cache.cc:5-39): per head h the
    cache is [K L x 64 | V L x 64]; the new k = qkv[1024 + 64h:], v =
    qkv[1536 + 64h:] become row L.  prior: uint16 [8 * 2 * L * 64]."""
    length = prior.size // (HKV * 2 * D)
    old = prior.reshape(HKV, 2, length, D)
    new = np.empty((HKV, 2, length + 1, D), dtype=prior.dtype)
    new[:, :, :length] = old
    new[:, 0, length] = qkv[1024:1536].reshape(HKV, D)
    new[:, 1, length] = qkv[1536:2048].reshape(HKV, D)
    return new.reshape(-1)


def ref_fixed64_cache(keys: np.ndarray, values: np.ndarray) -> np.ndarray:
    """Fixed-capacity cache of lfm25_attention_fixed64_head
    (experiments/kernels/lfm25_attention_fixed64_head.cc:25-57): per head
    [length as bf16, 0, K 64 x 64, V 64 x 64]; keys/values uint16 [8, T, 64]."""
    t = keys.shape[1]
    cache = np.zeros((HKV, 2 + 2 * 64 * D), dtype=np.uint16)
    cache[:, 0] = float_to_bf16_bits(np.float32(t))
    cache[:, 2: 2 + t * D] = keys.reshape(HKV, -1)
    cache[:, 2 + 64 * D: 2 + 64 * D + t * D] = values.reshape(HKV, -1)
    return cache.reshape(-1)


def ref_chunked_cache(keys: np.ndarray, values: np.ndarray, block_count: int) -> np.ndarray:
    """Chunked cache of lfm25_attention_chunked_head
    (experiments/kernels/lfm25_attention_chunked_head.cc:26-47): block_count
    blocks x 8 heads x [length-in-block as bf16, 0, K 64 x 64, V 64 x 64]."""
    t = keys.shape[1]
    cache = np.zeros((block_count, HKV, 2 + 2 * 64 * D), dtype=np.uint16)
    for j in range(block_count):
        n = max(0, min(64, t - 64 * j))
        cache[j, :, 0] = float_to_bf16_bits(np.float32(n))
        if n:
            cache[j, :, 2: 2 + n * D] = keys[:, 64 * j: 64 * j + n].reshape(HKV, -1)
            cache[j, :, 2 + 64 * D: 2 + 64 * D + n * D] = values[:, 64 * j: 64 * j + n].reshape(HKV, -1)
    return cache.reshape(-1)


def ref_packed_tail(hidden: np.ndarray, context: np.ndarray) -> np.ndarray:
    """[hidden 1024 | context 1024] (lfm25_attention_context_cache_kernel.py:64-67)."""
    return np.concatenate([hidden.reshape(-1), context.reshape(-1)])


def float_to_bf16_bits(x) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 numpy bit patterns."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(BF16)
