"""Hugging Face adapter: Lfm2ForCausalLM decodes on the paged B200 path unchanged.

The reference's CPU path is transformers' Lfm2Attention with a DynamicCache
(experiments/006_lfm25_baseline.py:115-127, experiments/010_cpu_greedy.py:43-63):
Lfm2Attention.forward (modeling_lfm2.py:244-281) normalises and rotates q/k,
calls `past_key_values.update(k, v, layer_idx)` (DynamicLayer.update,
cache_utils.py:102-120, a torch.cat of the whole cache per token) and then the
registered attention function.  This module plugs into exactly those two
calls:

  * `B200PagedCache` — a DynamicCache whose full-attention layers are
    `PagedAttentionLayer`s over one PagedKVCache (64-token bf16 blocks).
    update() records the new k/v and the sequence length and returns them;
    nothing is concatenated.  The conv layers stay transformers' own
    LinearAttentionLayer.
  * `paged_attention` — the attention function, registered under the name
    "b200_paged" (`AttentionInterface`).  With one new token it runs the fused
    decode-step kernel (b2_decode_step, mode B2_STORE_KV: the k/v append and
    the split-KV attention in one launch; q/k are already normalised and
    rotated by transformers); with a chunk of tokens it runs b2_prefill_append
    + b2_prefill_attn (tcgen05 tiles, causal within the chunk).

Usage:
    register()
    model.set_attn_implementation("b200_paged")     # or config._attn_implementation
    cache = B200PagedCache(model.config, max_batch_size=B, max_cache_len=N, device="cuda")
    model(ids, past_key_values=cache, use_cache=True)  /  model.generate(..., past_key_values=cache)

Batches must be unpadded (every row at the same position); a padded batch is
rejected with ValueError because the paged cache would otherwise attend to the
pad tokens.  The mask interface is left unregistered, so transformers builds no
4-D mask; causality comes from the cache lengths.
"""
from __future__ import annotations

import threading

import torch

from . import _lib
from .attention import D, HKV, HQ, choose_blocks_per_split, decode_step, num_splits_for, prefill
from .paged_cache import PagedKVCache, blocks_for

NAME = "b200_paged"
_pending = threading.local()


def _transformers():
    try:
        from transformers import AttentionInterface
        from transformers.cache_utils import CacheLayerMixin, DynamicCache
    except ImportError as e:   # the adapter is optional; the kernels do not need transformers
        raise ImportError("the Hugging Face adapter needs transformers") from e
    return AttentionInterface, CacheLayerMixin, DynamicCache


def register() -> None:
    """Register `paged_attention` as attention implementation "b200_paged"."""
    AttentionInterface, _, _ = _transformers()
    AttentionInterface.register(NAME, paged_attention)


_, _CacheLayerMixin, _DynamicCache = _transformers()


class PagedAttentionLayer(_CacheLayerMixin):
    """One full-attention layer of a B200PagedCache: index `att` into the pool's
    layers.  Tracks the cached length (the same for every row of the batch)."""

    is_sliding = False
    is_compileable = False

    def __init__(self, owner: "B200PagedCache", att: int, layer_idx: int):
        super().__init__()
        self.owner, self.att, self.layer_idx = owner, att, layer_idx
        self.length = 0
        self.is_initialized = True
        self.device, self.dtype = owner.device, torch.bfloat16

    def lazy_initialization(self, *args, **kwargs) -> None:
        pass

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        """Record the new k/v [B, 8, T, 64] for the attention call that follows;
        the attention function appends them to the pool."""
        b, h, t, d = key_states.shape
        if h != HKV or d != D or tuple(value_states.shape) != (b, h, t, d):
            raise ValueError(f"expected k/v [batch, {HKV}, tokens, {D}], got {tuple(key_states.shape)}")
        if b != self.owner.batch:
            raise ValueError(f"cache was built for batch {self.owner.batch}, got {b}")
        if self.length + t > self.owner.max_cache_len:
            raise ValueError(f"KV capacity {self.owner.max_cache_len} exceeded")
        _pending.item = (self, self.length, t, key_states)
        self.length += t
        return key_states, value_states

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        return self.length + query_length, 0

    def get_seq_length(self) -> int:
        return self.length

    def get_max_cache_shape(self) -> int:
        return self.owner.max_cache_len

    def reset(self) -> None:
        self.length = 0

    def reorder_cache(self, beam_idx: torch.LongTensor) -> None:
        raise NotImplementedError("beam search is not supported by the paged B200 cache")

    def crop(self, max_length: int) -> None:
        if max_length < 0:
            max_length = self.length + max_length
        self.length = max(0, min(self.length, max_length))


class B200PagedCache(_DynamicCache):
    """transformers Cache with the full-attention layers in a paged B200 pool.

    max_batch_size sequences of up to max_cache_len tokens each; the blocks of
    every sequence are reserved up front (64-token blocks, optionally handed
    out in shuffled order)."""

    def __init__(self, config, *, max_batch_size: int, max_cache_len: int, device="cuda",
                 shuffle_seed: int | None = None, blocks_per_split: int | None = None):
        super().__init__(config=config)
        text = config.get_text_config(decoder=True)
        if (text.num_attention_heads, text.num_key_value_heads, text.hidden_size // text.num_attention_heads) != \
                (HQ, HKV, D):
            raise ValueError("the B200 kernels are built for 16 query heads, 8 KV heads, head_dim 64")
        self.device = torch.device(device)
        self.batch = max_batch_size
        self.capacity = max_cache_len
        att_layers = [i for i, t in enumerate(text.layer_types) if t == "full_attention"]
        per_seq = blocks_for(max_cache_len)
        self.pool = PagedKVCache(max_batch_size * per_seq, max_cache_len, num_layers=len(att_layers),
                                 device=self.device, shuffle_seed=shuffle_seed)
        for _ in range(max_batch_size):
            self.pool.add_sequence(0, capacity=max_cache_len)
        self.tables = self.pool.block_tables()
        for a, i in enumerate(att_layers):
            self.layers[i] = PagedAttentionLayer(self, a, i)
        if blocks_per_split is None:
            blocks_per_split = choose_blocks_per_split(max_batch_size, max_batch_size * per_seq, fused=True)
        self.bps = blocks_per_split
        splits = num_splits_for(self.tables.shape[1], blocks_per_split)
        dev = self.device
        self.part_ml = torch.empty(max_batch_size * splits * HQ * 2, dtype=torch.float32, device=dev)
        self.part_o = torch.empty(max_batch_size * splits * HQ * D, dtype=torch.float32, device=dev)
        self.counters = torch.zeros(2 + HKV * max_batch_size, dtype=torch.int32, device=dev)
        self.dev_err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.past = torch.zeros(max_batch_size, dtype=torch.int32, device=dev)
        self._past_value = 0

    @property
    def max_batch_size(self) -> int:
        return self.batch

    @property
    def max_cache_len(self) -> int:
        return self.capacity

    def _past_lens(self, length: int) -> torch.Tensor:
        if self._past_value != length:
            self.past.fill_(length)
            self._past_value = length
        return self.past

    def check(self) -> None:
        """Raise RuntimeError if a kernel flagged a device error."""
        word = int(self.dev_err.item())
        if word:
            self.dev_err.zero_()
            self.counters.zero_()
            raise RuntimeError("paged attention device error: " + "; ".join(_lib.decode_dev_err(word)))


def paged_attention(module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                    attention_mask, scaling: float | None = None, dropout: float = 0.0, **kwargs):
    """transformers attention function over a B200PagedCache.  query [B, 16, T, 64],
    key/value [B, 8, T, 64] (normalised and rotated); returns ([B, T, 16, 64], None)."""
    item = getattr(_pending, "item", None)
    _pending.item = None
    # the key tensor is the one the paged layer's update() returned just before
    if item is None or item[3] is not key or item[0].layer_idx != getattr(module, "layer_idx", None):
        raise ValueError('attention implementation "b200_paged" needs past_key_values=B200PagedCache(...)')
    layer, past, t, _ = item
    cache = layer.owner
    b = query.shape[0]
    if dropout:
        raise ValueError("dropout is not supported")
    if tuple(query.shape) != (b, HQ, t, D):
        raise ValueError(f"expected query [batch, {HQ}, {t}, {D}], got {tuple(query.shape)}")
    pos = kwargs.get("position_ids")
    if pos is not None:
        want = torch.arange(past, past + t, device=pos.device)
        if pos.dim() != 2 or not bool((pos == want).all()):
            raise ValueError("padded or shifted positions are not supported by the paged B200 cache")
    scale = D ** -0.5 if scaling is None else float(scaling)
    # one row per token: [q 16x64 | k 8x64 | v 8x64], the layout the kernels read
    qkv = torch.cat([query.transpose(1, 2).reshape(b, t, HQ * D), key.transpose(1, 2).reshape(b, t, HKV * D),
                     value.transpose(1, 2).reshape(b, t, HKV * D)], dim=-1).to(torch.bfloat16)
    kp, vp = cache.pool.pool(layer.att)
    past_lens = cache._past_lens(past)
    if t == 1:
        out = torch.empty(b, 1, HQ, D, dtype=torch.bfloat16, device=query.device)
        decode_step(qkv[:, 0], past_lens, k_pool=kp, v_pool=vp, block_tables=cache.tables,
                    blocks_per_split=cache.bps, out=out, part_ml=cache.part_ml, part_o=cache.part_o,
                    counters=cache.counters, dev_err=cache.dev_err, mode=_lib.B2_STORE_KV, scale=scale)
        return out, None
    out = prefill(qkv.contiguous(), past_lens, k_pool=kp, v_pool=vp, block_tables=cache.tables, gamma_q=None,
                  gamma_k=None, cos=None, sin=None, dev_err=cache.dev_err, scale=scale, mode=_lib.B2_STORE_KV)
    return out, None
