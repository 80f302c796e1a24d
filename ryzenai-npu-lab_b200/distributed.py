"""Multi-GPU decode attention: sequence sharding and long-context split-KV.

One process per GPU (torch.distributed, NCCL over NVLink on B200; gloo works
for the host-side logic on CPU).  The reference has no multi-device code: its
long contexts stream 64-token blocks through one NPU core
(experiments/lfm25_attention_chunked_cache_kernel.py:21-89) and its x8 engine
splits heads over the 8 cores of one device (experiments/lfm25_x8.py:467-484).

Two modes:
  * batched decode (config C3): whole sequences are assigned to GPUs, balanced
    by token count (`shard_sequences`); there is no collective on the data
    path, each rank decodes its own sequences.
  * long context (config C4): the tokens of one sequence are split along the
    token axis (`token_ranges`); every rank computes a partial softmax state
    (max, sum, output) of the new query over its tokens, the states are
    all-gathered (16 x 66 fp32 = 4224 bytes per rank) and merged with the same
    log-sum-exp kernel that merges the splits inside one GPU.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .attention import BLOCK, D, EPS, HQ, choose_blocks_per_split, decode_step, merge_states, num_splits_for
from .paged_cache import PagedKVCache, blocks_for
from .rope import rope_table

STATE_FLOATS = 2 + D   # (max, sum) + 64 output values per query head


def shard_sequences(lengths: list[int], world: int) -> list[list[int]]:
    """Assign sequence indices to `world` ranks, balancing cached tokens:
    longest first, each to the rank with the fewest tokens so far (LPT)."""
    if world <= 0:
        raise ValueError("world must be positive")
    load = [0] * world
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda k: (-lengths[k], k)):
        r = min(range(world), key=lambda k: (load[k], k))
        shards[r].append(i)
        load[r] += lengths[i] + 1
    return [sorted(s) for s in shards]


def token_ranges(total: int, world: int) -> list[tuple[int, int]]:
    """Split tokens [0, total) into `world` contiguous ranges that start on
    64-token block boundaries (the last range takes the remainder)."""
    if world <= 0 or total < 0:
        raise ValueError("bad arguments")
    nblk = blocks_for(total)
    per = nblk // world
    extra = nblk % world
    out, start = [], 0
    for r in range(world):
        nb = per + (1 if r < extra else 0)
        end = min(total, start + nb * BLOCK)
        out.append((start, end))
        start = end
    return out


def gather_states(state: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather one state buffer per rank into [world, *state.shape]
    (one NCCL all-gather over NVLink; gloo on CPU)."""
    world = dist.get_world_size(group)
    out = torch.empty((world, *state.shape), dtype=state.dtype, device=state.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, state.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), state.contiguous(), group=group)
    return out


class LongContextDecode:
    """One sequence whose KV cache is split along the token axis over the ranks
    of `group`.  Rank r holds tokens token_ranges(capacity)[r] in its own
    paged pool; new tokens are appended on the last rank.  step() returns the
    bf16 context [16, 64] on every rank."""

    def __init__(self, capacity: int, gamma_q: torch.Tensor, gamma_k: torch.Tensor, *, group=None,
                 device: torch.device | str = "cuda", blocks_per_split: int | None = None, eps: float = EPS,
                 growth: int = 4096):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device)
        self.capacity = capacity
        self.ranges = token_ranges(capacity, self.world)
        self.start, self.end = self.ranges[self.rank]
        self.is_tail = self.rank == self.world - 1
        local_cap = (self.end - self.start) + (growth if self.is_tail else 0)
        local_cap = max(local_cap, 1)
        self.cache = PagedKVCache(blocks_for(local_cap), local_cap, device=self.device)
        self.cache.add_sequence(0)
        self.tables = self.cache.block_tables()
        self.local_len = 0
        self.eps = eps
        if blocks_per_split is None:
            blocks_per_split = choose_blocks_per_split(1, blocks_for(self.end - self.start + 1), fused=True)
        self.bps = blocks_per_split
        self.gamma_q = gamma_q.to(self.device, torch.bfloat16).contiguous()
        self.gamma_k = gamma_k.to(self.device, torch.bfloat16).contiguous()
        cos, sin = rope_table(capacity + growth + 1, device=self.device)
        # RoPE rows are looked up at the local slot; offset the table by this
        # rank's first global token so that the row is the global position.
        self.cos_all, self.sin_all = cos, sin
        splits = num_splits_for(self.cache.max_blocks, self.bps)
        self.splits = splits
        self.q = torch.empty(1, HQ, D, dtype=torch.bfloat16, device=self.device)
        self.part_ml = torch.empty(1, splits, HQ, 2, dtype=torch.float32, device=self.device)
        self.part_o = torch.empty(1, splits, HQ, D, dtype=torch.float32, device=self.device)
        # the exchanged state, [ml 16 x 2 | o 16 x 64] fp32, written in place by
        # the decode step and all-gathered as one buffer
        self.state = torch.empty(HQ * STATE_FLOATS, dtype=torch.float32, device=self.device)
        self.state_ml = self.state[: HQ * 2].view(1, HQ, 2)
        self.state_o = self.state[HQ * 2:].view(1, HQ, D)
        self.out = torch.empty(1, HQ, D, dtype=torch.bfloat16, device=self.device)
        self.dev_err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.counters = torch.zeros(2 + 8, dtype=torch.int32, device=self.device)
        self.past = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.seq = torch.zeros(1, dtype=torch.int32, device=self.device)

    def load_history(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """k, v: [8, L, 64] of the whole sequence (only this rank's range is kept)."""
        total = k.shape[1]
        lo, hi = self.start, min(self.end, total)
        if self.is_tail:
            hi = total
        n = max(0, hi - lo)
        if n:
            self.cache.write_dense(0, 0, k[:, lo:hi], v[:, lo:hi])
        self.local_len = n
        self.global_len = total

    def fill_random(self, total: int, generator: torch.Generator) -> None:
        """Synthetic history of `total` tokens, K/V ~ N(0, 1): this rank's range only."""
        kp, vp = self.cache.pool(0)
        kp.normal_(generator=generator)
        vp.normal_(generator=generator)
        lo, hi = self.start, min(self.end, total)
        if self.is_tail:
            hi = total
        self.local_len = max(0, hi - lo)
        self.global_len = total

    def set_lengths(self, global_len: int) -> None:
        """Place the state for a decode step at global position global_len
        (host copy of two int32; call outside CUDA graph capture)."""
        lo = self.start
        self.global_len = global_len
        if self.is_tail:
            self.local_len = global_len - lo
        self.past.fill_(global_len - lo)                       # slot (tail) / RoPE row offset
        self.seq.fill_(self.local_len + (1 if self.is_tail else 0))

    def step(self, qkv: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """qkv: bf16 [1, >= 2048] raw projections of the new token.  Lengths come
        from set_lengths(); the call is capturable in a CUDA graph (NCCL included)."""
        self.partial(qkv, stream)
        return self.merge(stream)

    def partial(self, qkv: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
        """This rank's part, one fused launch (b2_decode_step): q/k norm + RoPE at
        the global position (and the append on the last rank), split-KV
        attention over the local tokens, merged into one local fp32 state."""
        mode = _lib.B2_NORM_QK | _lib.B2_ROPE_QK | (_lib.B2_STORE_KV if self.is_tail else 0)
        kp, vp = self.cache.pool(0)
        # RoPE rows are read at past_lens; offsetting the table by this rank's
        # first global token turns the local slot into the global position.
        decode_step(qkv, self.past, k_pool=kp, v_pool=vp, block_tables=self.tables, blocks_per_split=self.bps,
                    out=None, part_ml=self.part_ml, part_o=self.part_o, counters=self.counters,
                    dev_err=self.dev_err, gamma_q=self.gamma_q, gamma_k=self.gamma_k,
                    cos=self.cos_all[self.start:], sin=self.sin_all[self.start:], q_out=self.q,
                    seq_lens=None if self.is_tail else self.seq, state_ml=self.state_ml, state_o=self.state_o,
                    mode=mode, eps=self.eps, stream=stream)

    def merge(self, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """Exchange the local states (one all-gather) and merge them into the context."""
        allst = gather_states(self.state, self.group)            # [world, 16 * 66]
        merge_states(allst, self.world, 1, out=self.out, stream=stream)
        return self.out[0]

    def check(self) -> None:
        word = int(self.dev_err.item())
        if word:
            self.dev_err.zero_()
            self.counters.zero_()
            raise RuntimeError("long-context decode device error: " + "; ".join(_lib.decode_dev_err(word)))
