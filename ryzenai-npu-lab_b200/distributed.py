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
    (max, sum, output) of the new query over its tokens and the states are
    merged.  Two exchanges: "p2p" (default on one host, one GPU per rank) —
    one kernel, b2_exchange_merge, writes the state into every rank's
    exchange area over NVLink, waits for the others' and merges, no
    collective library; "collective" — an all-gather (16 x 66 fp32 = 4224
    bytes per rank; NCCL, or gloo on CPU) and the log-sum-exp merge kernel.
"""
from __future__ import annotations

import ctypes
import socket

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


def p2p_possible(hosts: list[str], devices: list[str]) -> bool:
    """The P2P exchange needs every rank on one host and on its own GPU (its
    kernel waits for the other ranks; two ranks on one GPU could deadlock)."""
    return len(set(hosts)) == 1 and len(set(devices)) == len(devices) and 1 < len(devices) <= _lib.B2_XCHG_MAX_WORLD


def agree(failure: str | None, group=None) -> list[str]:
    """Every rank's failure text (None when it succeeded), on every rank: one
    all_gather_object, so that all ranks take the same branch afterwards."""
    outcomes: list[str | None] = [None] * dist.get_world_size(group)
    dist.all_gather_object(outcomes, failure, group=group)
    return [f"rank {r}: {o}" for r, o in enumerate(outcomes) if o]


def agree_device_errors(word: int, group=None) -> list[str]:
    """Every rank's device error word, on every rank (one all_gather_object):
    the ranks whose kernels flagged an error, with the decoded bits.  An empty
    list on every rank when none did, so all ranks take the same branch."""
    text = "; ".join(_lib.decode_dev_err(word)) if word else None
    return agree(text, group)


def open_peer_areas(entries: list, rank: int, open_fn, close_fn, group=None) -> tuple[list, list]:
    """Map every other rank's exchange area; `entries[r]` is what open_fn needs
    for rank r, and open_fn returns the mapped pointer.  The ranks agree on
    the outcome: if any rank fails, every rank unmaps what it mapped and all
    raise ValueError together (instead of the others waiting in the next
    collective for a rank that gave up)."""
    opened, ptrs, failure = [], [], None
    for r, entry in enumerate(entries):
        if r == rank:
            ptrs.append(None)
            continue
        try:
            ptr = open_fn(entry)
        except Exception as e:  # noqa: BLE001 - reported to every rank below
            failure = f"mapping rank {r}'s area: {e}"
            break
        opened.append((ptr, entry))
        ptrs.append(ptr)
    failed = agree(failure, group)
    if failed:
        for ptr, entry in opened:
            try:
                close_fn(ptr, entry)
            except Exception:  # noqa: BLE001 - already failing; keep unmapping the rest
                pass
        raise ValueError("P2P exchange setup failed: " + "; ".join(failed))
    return opened, ptrs


class PeerExchange:
    """Exchange areas for b2_exchange_merge: one in this rank's memory, the
    other ranks' mapped through CUDA IPC (peer access over NVLink).  All ranks
    of `group` construct it together; close() together.  A setup failure on
    any rank is a ValueError on every rank."""

    def __init__(self, batch: int, group=None, device: torch.device | str = "cuda"):
        lib = _lib.load()
        self.lib, self.group = lib, group
        self.device = torch.device(device)
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.batch = batch
        nbytes = lib.b2_exchange_bytes(self.world, batch)
        if nbytes <= 0:
            raise ValueError(f"exchange of world {self.world}, batch {batch} is not supported")
        self.area = torch.zeros(nbytes // 4, dtype=torch.int32, device=self.device)
        handle = ctypes.create_string_buffer(64)
        offset = ctypes.c_int64(0)
        failure = None
        if lib.b2_ipc_handle(ctypes.c_void_p(self.area.data_ptr()), handle, ctypes.byref(offset)) != _lib.B2_OK:
            failure = "b2_ipc_handle: " + _lib.last_error()
        uuid = str(torch.cuda.get_device_properties(self.device).uuid)
        info = [None] * self.world
        dist.all_gather_object(info, (handle.raw, offset.value, socket.gethostname(), uuid, failure), group=group)
        failed = [f"rank {r}: {i[4]}" for r, i in enumerate(info) if i[4]]
        if failed:
            raise ValueError("P2P exchange setup failed: " + "; ".join(failed))
        if not p2p_possible([i[2] for i in info], [i[3] for i in info]):
            raise ValueError("the P2P exchange needs all ranks on one host, each on its own GPU")

        def open_fn(entry):
            peer = ctypes.c_void_p()
            _lib.check(lib.b2_ipc_open(entry[0], entry[1], ctypes.byref(peer)), "b2_ipc_open")
            return peer.value

        def close_fn(ptr, entry):
            _lib.check(lib.b2_ipc_close(ctypes.c_void_p(ptr), entry[1]), "b2_ipc_close")

        opened, ptrs = open_peer_areas(info, self.rank, open_fn, close_fn, group)
        self.opened = [(ptr, entry[1]) for ptr, entry in opened]
        ptrs[self.rank] = self.area.data_ptr()
        self.areas = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=group)

    def merge(self, state_ml: torch.Tensor, state_o: torch.Tensor, out: torch.Tensor, dev_err: torch.Tensor,
              stream: torch.cuda.Stream | None = None) -> None:
        """This rank's state in, the world-merged bf16 context out (one launch)."""
        from .attention import _ptr, _stream
        rc = self.lib.b2_exchange_merge(_ptr(state_ml), _ptr(state_o), self.batch, self.areas, self.world,
                                        self.rank, _ptr(out), _ptr(dev_err), _stream(self.device, stream))
        _lib.check(rc, "b2_exchange_merge")

    def reset(self) -> None:
        """Zero the area after a device error (every rank together).  The first
        barrier makes sure no rank's exchange kernel is still writing tagged
        words into this area when it is cleared; the second, that no rank
        starts its next exchange before every area is clear."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.area.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for ptr, off in self.opened:
            _lib.check(self.lib.b2_ipc_close(ctypes.c_void_p(ptr), off), "b2_ipc_close")
        self.opened = []


class LongContextDecode:
    """One sequence whose KV cache is split along the token axis over the ranks
    of `group`.  Rank r holds tokens token_ranges(capacity)[r] in its own
    paged pool; new tokens are appended on the last rank.  step() returns the
    bf16 context [16, 64] on every rank.

    exchange: "p2p" (b2_exchange_merge over NVLink peer memory), "collective"
    (all-gather + merge kernel) or "auto" (p2p when the ranks are on distinct
    GPUs of one host with NCCL as the backend, else collective).  A world of
    one writes the context directly."""

    def __init__(self, capacity: int, gamma_q: torch.Tensor, gamma_k: torch.Tensor, *, group=None,
                 device: torch.device | str = "cuda", blocks_per_split: int | None = None, eps: float = EPS,
                 growth: int = 4096, exchange: str = "auto", max_ctas: int = 0):
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
        self.max_ctas = max_ctas
        if exchange not in ("auto", "p2p", "collective"):
            raise ValueError("exchange must be auto, p2p or collective")
        self.peer = None
        if self.world > 1 and exchange != "collective" and self.device.type == "cuda":
            if exchange == "p2p":
                self.peer = PeerExchange(1, group, self.device)
            elif dist.get_backend(group) == "nccl":
                try:
                    self.peer = PeerExchange(1, group, self.device)
                except ValueError:
                    self.peer = None
        elif exchange == "p2p":
            raise ValueError("the P2P exchange needs CUDA devices and a world of more than one")
        self.exchange = "p2p" if self.peer is not None else ("direct" if self.world == 1 else "collective")

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
        from set_lengths(); the call is capturable in a CUDA graph (NCCL included).
        With the P2P exchange the whole step is one call (b2_decode_step_exchange):
        the step kernel, then the combine kernel merging this rank's splits and
        exchanging the result with the other ranks over peer memory."""
        if self.exchange == "p2p":
            self._run(qkv, stream, exchange=(self.peer.areas, self.world, self.rank))
            return self.out[0]
        self.partial(qkv, stream)
        return self.merge(stream)

    def partial(self, qkv: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
        """This rank's part, one fused launch (b2_decode_step): q/k norm + RoPE at
        the global position (and the append on the last rank), split-KV
        attention over the local tokens, merged into one local fp32 state (the
        context itself for a world of one)."""
        self._run(qkv, stream)

    def _run(self, qkv: torch.Tensor, stream: torch.cuda.Stream | None, exchange=None) -> None:
        mode = _lib.B2_NORM_QK | _lib.B2_ROPE_QK | (_lib.B2_STORE_KV if self.is_tail else 0)
        kp, vp = self.cache.pool(0)
        # RoPE rows are read at past_lens; offsetting the table by this rank's
        # first global token turns the local slot into the global position.
        direct = self.exchange == "direct" or exchange is not None
        decode_step(qkv, self.past, k_pool=kp, v_pool=vp, block_tables=self.tables, blocks_per_split=self.bps,
                    out=self.out if direct else None, part_ml=self.part_ml, part_o=self.part_o,
                    counters=self.counters, dev_err=self.dev_err, gamma_q=self.gamma_q, gamma_k=self.gamma_k,
                    cos=self.cos_all[self.start:], sin=self.sin_all[self.start:], q_out=self.q,
                    seq_lens=None if self.is_tail else self.seq,
                    state_ml=None if direct else self.state_ml, state_o=None if direct else self.state_o,
                    mode=mode, eps=self.eps, max_ctas=self.max_ctas, stream=stream, exchange=exchange)

    def merge(self, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """Exchange the local states and merge them into the context: one P2P
        kernel, or an all-gather and the merge kernel (nothing for a world of one)."""
        if self.exchange == "p2p":
            self.peer.merge(self.state_ml, self.state_o, self.out, self.dev_err, stream)
        elif self.exchange == "collective":
            allst = gather_states(self.state, self.group)            # [world, 16 * 66]
            merge_states(allst, self.world, 1, out=self.out, stream=stream)
        return self.out[0]

    def close(self) -> None:
        """Release the peer mappings (every rank together)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def check(self) -> None:
        """Synchronise on the device error word.  With several ranks the words
        are agreed first (every rank calls check() together), so that all
        ranks raise together and can then reset_exchange() together."""
        word = int(self.dev_err.item())
        failed = agree_device_errors(word, self.group) if self.world > 1 else (
            [f"rank 0: {'; '.join(_lib.decode_dev_err(word))}"] if word else [])
        if failed:
            self.dev_err.zero_()
            self.counters.zero_()
            raise RuntimeError("long-context decode device error: " + "; ".join(failed) +
                               ("; call reset_exchange() on every rank" if self.peer is not None else ""))

    def reset_exchange(self) -> None:
        """After a device error in the P2P exchange: zero the areas (every rank)."""
        if self.peer is not None:
            self.peer.reset()
