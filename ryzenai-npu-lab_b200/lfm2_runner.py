"""Whole-token LFM2.5-230M decode runner around the paged decode-attention path.

The API mirrors the reference's x8 decode loop, X8Model
(experiments/lfm25_x8_model.py:64-148): reset(), step(token_ids, select),
prefill(ids), kv(att_index, position) — for a batch of sequences instead of
one.  Like the x8 engine's one submission per token
(experiments/lfm25_x8.py:227-313, README.md:83-85), a whole token (14 layers
and the head) is one CUDA-graph replay.

The attention layers' hot path — q/k RMSNorm + RoPE + paged KV append +
split-KV attention — runs in libb2attn.so's fused decode step.  Around it
(fused_glue=True, the default) the residual adds + RMSNorms, the SwiGLU gate
and the short-convolution step are libb2attn.so kernels too (b2_add_rmsnorm,
b2_swiglu, b2_shortconv_step); fused_glue=False runs that glue as plain
torch ops.  The projections are cuBLAS GEMMs (torch.matmul, w1 and w3
stacked into one) by default; own_gemm=True runs them on libb2attn.so's
tensor-core GEMM (b2_gemm, with the SwiGLU gate as the epilogue of the
stacked w1/w3 product), which at batch 256 is 1.2-1.7x slower than cuBLAS per
projection.  With fused_glue=False and own_gemm=True the torch glue runs
around b2_gemm products, the w1/w3 product tiled as in the fused epilogue.
Both follow the model definition the reference's CPU path uses
(transformers modeling_lfm2.py: Lfm2RMSNorm 59-64, Lfm2MLP 135-152,
Lfm2ShortConv.slow_forward 356-387, Lfm2DecoderLayer.forward 413-442,
Lfm2Model.forward 483-538) and its cache update (cache_utils.py:771-786: the
3-token conv state rolls by one per token).

Weights come from a state dict with the Hugging Face parameter names
(model.layers.{i}.self_attn.q_proj.weight, ...), e.g. a random-init model.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _lib, block
from .attention import PagedDecodeAttention
from .paged_cache import PagedKVCache, blocks_for

LFM25_LAYER_TYPES = ("conv", "conv", "attention", "conv", "attention", "conv", "attention", "conv",
                     "attention", "conv", "attention", "conv", "attention", "conv")   # lfm25_x8.py:55-57


@dataclass(frozen=True)
class LFM2Config:
    hidden: int = 1024
    ffn: int = 2560
    vocab: int = 65536
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 64
    conv_l: int = 3
    eps: float = 1e-5
    layer_types: tuple = field(default=LFM25_LAYER_TYPES)

    @property
    def attention_layers(self) -> list[int]:
        return [i for i, t in enumerate(self.layer_types) if t == "attention"]

    @property
    def conv_layers(self) -> list[int]:
        return [i for i, t in enumerate(self.layer_types) if t == "conv"]


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Lfm2RMSNorm: weight * bf16(x * rsqrt(mean(x^2) + eps)), fp32 inside."""
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return weight * h.to(x.dtype)


class LFM2DecodeRunner:
    """Batched greedy decode of an LFM2.5-shaped model with paged KV."""

    def __init__(self, state_dict: dict, config: LFM2Config = LFM2Config(), *, max_batch: int,
                 max_context: int, device: torch.device | str = "cuda", use_graph: bool = True,
                 blocks_per_split: int | None = None, fused_glue: bool = True, own_gemm: bool = False):
        self.cfg = config
        self.device = torch.device(device)
        self.max_batch = max_batch
        self.max_context = max_context
        dev, bf = self.device, torch.bfloat16

        def w(name):
            return state_dict[name].to(dev, bf).contiguous()

        self.embed = w("model.embed_tokens.weight")
        self.final_norm = w("model.embedding_norm.weight")
        self.head = w("lm_head.weight") if "lm_head.weight" in state_dict else self.embed
        self.layers = []
        att_ids = {layer: a for a, layer in enumerate(config.attention_layers)}
        conv_ids = {layer: c for c, layer in enumerate(config.conv_layers)}
        for i, kind in enumerate(config.layer_types):
            p = f"model.layers.{i}."
            lw = {"kind": kind, "op_norm": w(p + "operator_norm.weight"), "ffn_norm": w(p + "ffn_norm.weight"),
                  "w1": w(p + "feed_forward.w1.weight"), "w3": w(p + "feed_forward.w3.weight"),
                  "w2": w(p + "feed_forward.w2.weight")}
            lw["w13"] = torch.cat([lw["w1"], lw["w3"]]).contiguous()      # [2 * ffn, hidden]
            if kind == "attention":
                lw["qkv"] = torch.cat([w(p + "self_attn.q_proj.weight"), w(p + "self_attn.k_proj.weight"),
                                       w(p + "self_attn.v_proj.weight")]).contiguous()
                lw["out"] = w(p + "self_attn.out_proj.weight")
                lw["q_gamma"] = w(p + "self_attn.q_layernorm.weight")
                lw["k_gamma"] = w(p + "self_attn.k_layernorm.weight")
                lw["att"] = att_ids[i]
            else:
                lw["in"] = w(p + "conv.in_proj.weight")
                lw["out"] = w(p + "conv.out_proj.weight")
                lw["conv"] = w(p + "conv.conv.weight")[:, 0, :].contiguous()   # [hidden, L]
                lw["conv_id"] = conv_ids[i]
            self.layers.append(lw)

        n_att = len(config.attention_layers)
        per_seq = blocks_for(max_context)
        self.cache = PagedKVCache(max_batch * per_seq, max_context, num_layers=n_att, device=dev)
        for _ in range(max_batch):
            self.cache.add_sequence(0, capacity=max_context)
        self.tables = self.cache.block_tables()
        self.attn = [PagedDecodeAttention(self.cache, lw["q_gamma"], lw["k_gamma"], max_batch, max_context + 1,
                                          eps=config.eps, blocks_per_split=blocks_per_split,
                                          work_blocks=max_batch * per_seq)
                     for lw in self.layers if lw["kind"] == "attention"]
        self.conv_state = torch.zeros(len(config.conv_layers), max_batch, config.hidden, config.conv_l,
                                      dtype=bf, device=dev)
        self.past = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self.seq = torch.ones(max_batch, dtype=torch.int32, device=dev)
        self.ids = torch.zeros(max_batch, dtype=torch.long, device=dev)
        self.next_ids = torch.zeros(max_batch, dtype=torch.long, device=dev)
        self.logits = torch.empty(max_batch, config.vocab, dtype=bf, device=dev)
        self.position = 0
        self.use_graph = use_graph and self.device.type == "cuda"
        self._graph = None
        self.fused_glue = fused_glue
        self.own_gemm = own_gemm
        self.gemm_err = torch.zeros(1, dtype=torch.int32, device=dev)
        if fused_glue:
            ffn = self.layers[0]["w1"].shape[0]
            hd = config.hidden

            def buf(*shape):
                return torch.empty(*shape, dtype=bf, device=dev)
            self.h, self.x, self.o, self.y = buf(max_batch, hd), buf(max_batch, hd), buf(max_batch, hd), \
                buf(max_batch, hd)
            self.qkv = buf(max_batch, (config.heads + 2 * config.kv_heads) * config.head_dim)
            self.bcx, self.gu, self.m = buf(max_batch, 3 * hd), buf(max_batch, 2 * ffn), buf(max_batch, ffn)

    # ---------------------------------------------------------------- model

    def _token(self) -> None:
        """One token for every sequence: ids -> logits, next_ids; advances past."""
        if self.fused_glue:
            self._token_fused()
        else:
            self._token_torch()

    def _mm(self, a: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> None:
        """out = a @ w.T: b2_gemm, or cuBLAS with own_gemm=False."""
        if self.own_gemm:
            block.gemm(a, w, out=out, dev_err=self.gemm_err)
        else:
            torch.matmul(a, w.t(), out=out)

    def _token_fused(self) -> None:
        """The token with the layer glue in libb2attn.so: per layer two GEMMs
        around the mixer (attention step or short-convolution step), then
        residual + RMSNorm, the stacked w1/w3 GEMM with the SwiGLU gate, the w2
        GEMM; each residual add is fused into the RMSNorm that follows it."""
        cfg, b = self.cfg, self.max_batch
        h, x, o = self.h, self.x, self.o
        torch.index_select(self.embed, 0, self.ids, out=h)
        torch.add(self.past, 1, out=self.seq)
        block.add_rmsnorm(h, None, self.layers[0]["op_norm"], cfg.eps, out=x)
        n = len(self.layers)
        for i, lw in enumerate(self.layers):
            if lw["kind"] == "attention":
                self._mm(x, lw["qkv"], self.qkv)                                    # [B, 2048]: q | k | v
                ctx = self.attn[lw["att"]].step(lw["att"], self.qkv, self.past, self.seq, self.tables)
                self._mm(ctx.reshape(b, cfg.heads * cfg.head_dim), lw["out"], o)
            else:
                self._mm(x, lw["in"], self.bcx)                                     # [B, 3 * hidden]: B | C | x
                block.shortconv_step(self.bcx, self.conv_state[lw["conv_id"]], lw["conv"], out=self.y)
                self._mm(self.y, lw["out"], o)
            block.add_rmsnorm(o, h, lw["ffn_norm"], cfg.eps, out=x, sum_out=h)  # h += mixer; x = ffn_norm(h)
            if self.own_gemm:
                block.gemm(x, lw["w13"], out=self.m, dev_err=self.gemm_err, swiglu=True)
            else:
                torch.matmul(x, lw["w13"].t(), out=self.gu)
                block.swiglu(self.gu, out=self.m)
            self._mm(self.m, lw["w2"], o)
            nxt = self.layers[i + 1]["op_norm"] if i + 1 < n else self.final_norm
            block.add_rmsnorm(o, h, nxt, cfg.eps, out=x, sum_out=h)             # h += ffn; x = next norm(h)
        self._mm(x, self.head, self.logits)
        block.argmax_rows(self.logits, out=self.next_ids)
        self.past.add_(1)

    def _proj(self, a: torch.Tensor, w: torch.Tensor, **tiling) -> torch.Tensor:
        """a @ w.T into a new tensor: b2_gemm, or cuBLAS with own_gemm=False."""
        if not self.own_gemm:
            return a @ w.t()
        out = torch.empty(a.shape[0], w.shape[0], dtype=a.dtype, device=a.device)
        return block.gemm(a, w, out=out, dev_err=self.gemm_err, **tiling)

    def _token_torch(self) -> None:
        """The token with the layer glue as torch ops."""
        cfg = self.cfg
        b = self.max_batch
        ffn = self.layers[0]["w1"].shape[0]
        # the w1/w3 product as the fused SwiGLU epilogue tiles it (same fp32 sums)
        t, sp, _ = block.gemm_plan(b, ffn, cfg.hidden, _lib.B2_GEMM_SWIGLU) if self.own_gemm else (0, 0, 0)
        h = self.embed[self.ids]                                   # [B, hidden]
        torch.add(self.past, 1, out=self.seq)
        for lw in self.layers:
            x = rms_norm(h, lw["op_norm"], cfg.eps)
            if lw["kind"] == "attention":
                qkv = self._proj(x, lw["qkv"])                      # [B, 2048]: q | k | v
                ctx = self.attn[lw["att"]].step(lw["att"], qkv, self.past, self.seq, self.tables)
                o = self._proj(ctx.reshape(b, cfg.heads * cfg.head_dim), lw["out"])
            else:
                bcx = self._proj(x, lw["in"])                       # [B, 3 * hidden]: B | C | x
                bg, cg, xg = bcx.split(cfg.hidden, dim=-1)
                bx = bg * xg
                st = self.conv_state[lw["conv_id"]]
                st.copy_(torch.cat([st[..., 1:], bx[..., None]], dim=-1))
                conv = torch.sum(st * lw["conv"], dim=-1)
                o = self._proj(cg * conv, lw["out"])
            h = o + h
            hn = rms_norm(h, lw["ffn_norm"], cfg.eps)
            if self.own_gemm:
                gu = self._proj(hn, lw["w13"], tile_n=t, splits=sp)
                g, u = gu[:, :ffn], gu[:, ffn:]
            else:
                g, u = hn @ lw["w1"].t(), hn @ lw["w3"].t()
            h = h + self._proj(torch.nn.functional.silu(g) * u, lw["w2"])
        h = rms_norm(h, self.final_norm, cfg.eps)
        if self.own_gemm:
            block.gemm(h, self.head, out=self.logits, dev_err=self.gemm_err)
        else:
            torch.matmul(h, self.head.t(), out=self.logits)
        torch.argmax(self.logits, dim=-1, out=self.next_ids)
        self.past.add_(1)

    def _run(self) -> None:
        if not self.use_graph:
            self._token()
            return
        if self._graph is None:
            # warm up on a side stream, then capture one token (state is
            # restored afterwards so the capture run does not count)
            saved = (self.past.clone(), self.conv_state.clone())  # restored after the capture run
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                self._token()
            torch.cuda.current_stream(self.device).wait_stream(s)
            self.past.copy_(saved[0])
            self.conv_state.copy_(saved[1])
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._token()
            self.past.copy_(saved[0])
            self.conv_state.copy_(saved[1])
            self._graph = g
        self._graph.replay()

    # ---------------------------------------------------------------- X8Model-like API

    def reset(self) -> None:
        """Forget every sequence (KV lengths and conv states back to zero)."""
        self.past.zero_()
        self.conv_state.zero_()
        self.position = 0

    def step(self, token_ids, select: bool = True):
        """Run one position for every sequence.  Returns the selected next token
        ids (int64 [B], on the device) when `select` is true, else None."""
        if self.position >= self.max_context:
            raise ValueError(f"KV capacity {self.max_context} reached")
        ids = torch.as_tensor(token_ids, dtype=torch.long).reshape(-1)
        if ids.numel() != self.max_batch:
            raise ValueError(f"expected {self.max_batch} token ids, got {ids.numel()}")
        self.ids.copy_(ids, non_blocking=True)
        self._run()
        self.position += 1
        return self.next_ids if select else None

    def prefill(self, token_ids):
        """Process prompt tokens [B, T] position by position; the last one also
        selects the next token (returned, int64 [B] on the device)."""
        ids = torch.as_tensor(token_ids, dtype=torch.long)
        for t in range(ids.shape[1]):
            out = self.step(ids[:, t], select=t == ids.shape[1] - 1)
        return out

    def generate(self, prompt_ids, new_tokens: int) -> torch.Tensor:
        """Greedy decode: prefill the prompts, then feed back the argmax."""
        nxt = self.prefill(prompt_ids)
        out = [nxt.clone()]
        for _ in range(new_tokens - 1):
            nxt = self.step(nxt)
            out.append(nxt.clone())
        return torch.stack(out, dim=1)

    def kv(self, att_index: int, seq: int, position: int):
        """(keys, values) [8, position + 1, 64] of one attention layer and sequence
        (experiments/lfm25_x8_model.py:85-92)."""
        return self.cache.read_dense(att_index, seq, position + 1)

    def check(self) -> None:
        for a in self.attn:
            a.check()
        word = int(self.gemm_err.item())
        if word:
            self.gemm_err.zero_()
            raise RuntimeError("b2_gemm device error: " + "; ".join(_lib.decode_dev_err(word)))
