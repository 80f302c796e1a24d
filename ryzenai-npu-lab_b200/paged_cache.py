"""Paged BF16 KV cache: block pools, a block allocator and block tables.

Replaces the reference's per-core cache buffers, which are copied whole on
every append (experiments/kernels/lfm25_attention_append_cache.cc:5-39) or
streamed at a fixed capacity tier (experiments/lfm25_x8.py:116-123,263-270;
experiments/lfm25_x8_model.py:22,139).

Layout per attention layer (the library's pool layout):
    k_pool, v_pool : bf16 [num_blocks, 8 kv heads, 64 tokens, 64 dims]
One (block, head) tile is 8 KiB contiguous, which is the unit the decode
kernel streams with one TMA box.  Token t of a sequence lives in pool block
block_table[t // 64], row t % 64.  All layers share the block tables (a
sequence owns the same block ids in every layer's pool).
"""
from __future__ import annotations

import torch

HKV, D, BLOCK = 8, 64, 64
BLOCK_BYTES = 2 * HKV * BLOCK * D * 2   # K + V tile bytes of one block, all heads: 128 KiB


def blocks_for(tokens: int) -> int:
    return (tokens + BLOCK - 1) // BLOCK


class BlockAllocator:
    """Free list of pool block ids (host side).  The order of the free list is
    shuffled with a seeded generator when `shuffle_seed` is given, so that a
    sequence's blocks are scattered over the pool like in a long-running server."""

    def __init__(self, num_blocks: int, shuffle_seed: int | None = None):
        if num_blocks <= 0:
            raise ValueError("num_blocks must be positive")
        self.num_blocks = num_blocks
        if shuffle_seed is None:
            order = list(range(num_blocks))
        else:
            g = torch.Generator().manual_seed(shuffle_seed)
            order = torch.randperm(num_blocks, generator=g).tolist()
        self._free = order[::-1]   # pop() hands out order[0], order[1], ...
        self._used: set[int] = set()

    @property
    def free(self) -> int:
        return len(self._free)

    def alloc(self, n: int) -> list[int]:
        if n < 0:
            raise ValueError("n must be >= 0")
        if n > len(self._free):
            raise MemoryError(f"KV pool exhausted: need {n} blocks, {len(self._free)} free")
        out = [self._free.pop() for _ in range(n)]
        self._used.update(out)
        return out

    def release(self, blocks) -> None:
        """Return blocks to the free list.  A block outside the pool, not
        handed out, or listed twice is refused (nothing is released): two
        sequences sharing a block would overwrite each other's keys."""
        blocks = list(blocks)
        for b in blocks:
            if not 0 <= b < self.num_blocks:
                raise ValueError(f"block {b} outside the pool")
            if b not in self._used:
                raise ValueError(f"block {b} is not allocated")
        if len(set(blocks)) != len(blocks):
            raise ValueError("a block is listed twice")
        self._used.difference_update(blocks)
        self._free.extend(blocks)


class PagedKVCache:
    """K/V pools for `num_layers` attention layers plus per-sequence block tables.

    capacity_tokens is the most tokens any sequence may hold; it fixes the
    block-table width (max_blocks_per_seq).  Sequences are registered with
    `add_sequence`, which allocates the blocks its capacity needs up front, so
    a decode step never allocates.
    """

    def __init__(self, num_blocks: int, capacity_tokens: int, num_layers: int = 1,
                 device: torch.device | str = "cuda", shuffle_seed: int | None = None,
                 fill: float | None = None):
        if capacity_tokens <= 0:
            raise ValueError("capacity_tokens must be positive")
        self.num_blocks = num_blocks
        self.num_layers = num_layers
        self.device = torch.device(device)
        self.max_blocks = blocks_for(capacity_tokens)
        shape = (num_layers, num_blocks, HKV, BLOCK, D)
        if fill is None:
            self.k = torch.empty(shape, dtype=torch.bfloat16, device=self.device)
            self.v = torch.empty(shape, dtype=torch.bfloat16, device=self.device)
        else:
            self.k = torch.full(shape, fill, dtype=torch.bfloat16, device=self.device)
            self.v = torch.full(shape, fill, dtype=torch.bfloat16, device=self.device)
        self.allocator = BlockAllocator(num_blocks, shuffle_seed)
        self._tables: list[list[int]] = []
        self.lengths: list[int] = []

    @property
    def batch(self) -> int:
        return len(self._tables)

    def add_sequence(self, length: int = 0, capacity: int | None = None) -> int:
        cap = self.max_blocks * BLOCK if capacity is None else capacity
        if not 0 <= length <= cap <= self.max_blocks * BLOCK:
            raise ValueError(f"length {length} / capacity {cap} outside [0, {self.max_blocks * BLOCK}]")
        self._tables.append(self.allocator.alloc(blocks_for(cap)))
        self.lengths.append(length)
        return len(self._tables) - 1

    def release_sequence(self, seq: int) -> None:
        """Return a finished sequence's blocks to the pool.  Its row stays (block
        tables keep their batch index) with no blocks and length 0: it must
        not be stepped again, since a row of -1 entries is a device error."""
        self.allocator.release(self._tables[seq])
        self._tables[seq] = []
        self.lengths[seq] = 0

    def block_tables(self) -> torch.Tensor:
        """int32 [batch, max_blocks_per_seq]; unused entries are -1."""
        t = torch.full((self.batch, self.max_blocks), -1, dtype=torch.int32)
        for i, row in enumerate(self._tables):
            t[i, : len(row)] = torch.tensor(row, dtype=torch.int32)
        return t.to(self.device)

    def table(self, seq: int) -> list[int]:
        return list(self._tables[seq])

    def pool(self, layer: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
        return self.k[layer], self.v[layer]

    def write_dense(self, layer: int, seq: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Copy a dense [8, T, 64] history into the sequence's blocks (set-up
        of synthetic caches and of the reference-layout shims; not the decode path)."""
        t = k.shape[1]
        if blocks_for(t) > len(self._tables[seq]):
            raise ValueError("history longer than the sequence's capacity")
        kp, vp = self.pool(layer)
        nb = blocks_for(t)
        if nb == 0:
            return
        ids = torch.tensor(self._tables[seq][:nb], device=self.device)
        pad = nb * BLOCK - t
        kd = torch.nn.functional.pad(k.to(self.device), (0, 0, 0, pad)).reshape(HKV, nb, BLOCK, D)
        vd = torch.nn.functional.pad(v.to(self.device), (0, 0, 0, pad)).reshape(HKV, nb, BLOCK, D)
        kp[ids] = kd.transpose(0, 1).to(torch.bfloat16)
        vp[ids] = vd.transpose(0, 1).to(torch.bfloat16)

    def read_dense(self, layer: int, seq: int, length: int) -> tuple[torch.Tensor, torch.Tensor]:
        """[8, length, 64] K and V of one sequence (the x8 runner's kv(),
        experiments/lfm25_x8_model.py:85-92)."""
        kp, vp = self.pool(layer)
        nb = blocks_for(length)
        ids = torch.tensor(self._tables[seq][:nb], device=self.device, dtype=torch.long)
        k = kp[ids].transpose(0, 1).reshape(HKV, nb * BLOCK, D)[:, :length]
        v = vp[ids].transpose(0, 1).reshape(HKV, nb * BLOCK, D)[:, :length]
        return k, v
