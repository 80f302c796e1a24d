"""A CPU model of how the fused decode step (csrc/b2_attn.cu: decode_step_impl,
producer_load, step_producer, step_merger) distributes its work and merges
splits across CTAs, checked under random interleavings of the CTAs.

Work items are (sequence b, split, kv head).  Batches of up to 512 sequences
with more than one split per sequence (block-table width > blocks per split)
enumerate only real items through a prefix sum of splits per sequence
(compact); the others walk the dense (split, sequence, head) space and skip
splits past a sequence's end (with one split per sequence there are none).
The prefix sum is formed as the producer warp forms it: 32-sequence chunks
in turn, each by a warp scan (shfl_up by 1, 2, 4, 8, 16) plus the running
total of the chunks before it.  CTA i takes item i first, then items
counter + gridDim from a global counter.  When a sequence has more than one
split, the merger warp of the CTA that finishes a split counts the arrival
for (b, kv head); the last of nsplit arrivals merges all splits and resets the
count to zero.

Claims: every real item is processed exactly once and nothing else; exactly
one merge per (sequence, kv head) with several splits, after all of its
splits' partial states were stored; all counters are zero afterwards (so the
next step needs no reset); the host's grid equalisation gives every CTA at
least one item.
"""
import math
import random

import pytest

HKV = 8
MAX_COMPACT = 512


def nsplits(seq_len: int, bps: int) -> int:
    return math.ceil(math.ceil(seq_len / 64) / bps)


def chunk_prefix(splits: list[int]) -> list[int]:
    """step_producer's prefix: prefix[b] = splits of sequences 0..b-1, from a
    Hillis-Steele warp scan of each 32-sequence chunk (lane = b % 32) and the
    running total of the chunks before it (the scan's lane 31)."""
    batch = len(splits)
    prefix = [0] * (batch + 1)
    running = 0
    for c0 in range(0, batch, 32):
        incl = [splits[c0 + lane] if c0 + lane < batch else 0 for lane in range(32)]
        off = 1
        while off < 32:
            incl = [incl[i] + (incl[i - off] if i >= off else 0) for i in range(32)]
            off *= 2
        for lane in range(32):
            if c0 + lane < batch:
                prefix[c0 + lane + 1] = running + incl[lane]
        running += incl[31]
    return prefix


def enumerate_items(lens: list[int], bps: int, max_blocks: int):
    """producer_load's decoding of work index w (returns total and a decoder)."""
    batch = len(lens)
    compact = batch <= MAX_COMPACT and math.ceil(max_blocks / bps) > 1
    if compact:
        prefix = chunk_prefix([nsplits(n, bps) for n in lens])
        total = prefix[-1] * HKV
    else:
        total = math.ceil(max_blocks / bps) * batch * HKV

    def decode(w):
        kvh, p = w & 7, w >> 3
        if compact:
            lo, hi = 0, batch                  # largest b with prefix[b] <= p
            while hi - lo > 1:
                mid = (lo + hi) // 2
                if prefix[mid] <= p:
                    lo = mid
                else:
                    hi = mid
            b, split = lo, p - prefix[lo]
        else:
            split, b = p // batch, p % batch
        if split >= nsplits(lens[b], bps):
            return None                        # dense enumeration: a split past the end
        return b, split, kvh

    return total, decode


def grid_size(total: int, sms: int, max_ctas: int = 0) -> int:
    """decode_step_impl's grid: 3 CTAs per SM (or max_ctas), equal waves."""
    ctas = sms * 3
    if 0 < max_ctas < ctas:
        ctas = max_ctas
    ctas = min(ctas, total)
    waves = math.ceil(total / ctas)
    return math.ceil(total / waves)


def simulate(lens, bps, max_blocks, sms, seed, max_ctas=0):
    rng = random.Random(seed)
    total, decode = enumerate_items(lens, bps, max_blocks)
    ctas = grid_size(total, sms, max_ctas)
    counter = 0
    arrivals = {}                              # (b, kvh) -> count (the device counters)
    stored = set()                             # partial states in memory
    processed = []
    merges = []
    first = list(range(ctas))                  # CTA i's first item is i
    alive = list(range(ctas))
    while alive:
        c = rng.choice(alive)
        if first[c] is not None:
            w, first[c] = first[c], None
        else:
            w = counter + ctas                 # atomicAdd(work_ctr, 1) + gridDim.x
            counter += 1
        if w >= total:
            alive.remove(c)
            continue
        item = decode(w)
        if item is None:
            continue
        b, split, kvh = item
        processed.append(item)
        ns = nsplits(lens[b], bps)
        if ns == 1:
            continue                           # a whole-sequence item writes its context itself
        stored.add(item)                       # the consumers' stores, released before the arrival
        k = (b, kvh)
        last = arrivals.get(k, 0) == ns - 1
        arrivals[k] = arrivals.get(k, 0) + 1
        if last:
            assert all((b, s, kvh) in stored for s in range(ns)), "merge before all partial states"
            merges.append(k)
            arrivals[k] = 0                    # atomicExch(cnt, 0)
    return total, ctas, processed, merges, arrivals


@pytest.mark.parametrize("seed", range(20))
def test_compact_batches_cover_every_item_once(seed):
    rng = random.Random(seed)
    batch = rng.choice([1, 3, 64, 300])
    lens = [rng.choice([0, 1, 63, 64, 65, rng.randint(1, 9000)]) for _ in range(batch)]
    lens = [n for n in lens if n > 0] or [1]            # empty sequences get no item (written apart)
    bps = rng.choice([1, 4, 12, 32, 64])
    max_blocks = max(math.ceil(n / 64) for n in lens)
    sms = rng.choice([1, 7, 148])
    total, ctas, processed, merges, arrivals = simulate(lens, bps, max_blocks, sms, seed)
    want = {(b, s, h) for b, n in enumerate(lens) for s in range(nsplits(n, bps)) for h in range(HKV)}
    assert len(processed) == len(set(processed)) and set(processed) == want
    assert total == len(want) and ctas <= total
    multi = {(b, h) for b, n in enumerate(lens) if nsplits(n, bps) > 1 for h in range(HKV)}
    assert len(merges) == len(set(merges)) and set(merges) == multi
    assert all(v == 0 for v in arrivals.values())


@pytest.mark.parametrize("seed", range(4))
def test_dense_batches_skip_splits_past_the_end(seed):
    rng = random.Random(100 + seed)
    batch = MAX_COMPACT + 1 + rng.randint(0, 200)
    lens = [rng.randint(1, 3000) for _ in range(batch)]
    bps = rng.choice([4, 16])
    max_blocks = max(math.ceil(n / 64) for n in lens) + rng.randint(0, 3)   # a table wider than needed
    total, ctas, processed, merges, arrivals = simulate(lens, bps, max_blocks, 148, seed)
    want = {(b, s, h) for b, n in enumerate(lens) for s in range(nsplits(n, bps)) for h in range(HKV)}
    assert len(processed) == len(set(processed)) and set(processed) == want
    assert total >= len(want)
    assert all(v == 0 for v in arrivals.values())


@pytest.mark.parametrize("total", [1, 7, 443, 444, 445, 520, 888, 5000, 123457])
@pytest.mark.parametrize("max_ctas", [0, 1, 100])
def test_equal_waves_leave_no_cta_idle(total, max_ctas):
    ctas = grid_size(total, 148, max_ctas)
    waves = math.ceil(total / ctas)
    assert 1 <= ctas <= total and ctas * (waves - 1) < total <= ctas * waves
    assert ctas <= (max_ctas if max_ctas > 0 else 444)


@pytest.mark.parametrize("batch", [1, 2, 8, 31, 32, 33, 64, 100, 255, 256, 257, 511, 512])
def test_chunk_scans_form_the_prefix_sum(batch):
    rng = random.Random(batch)
    splits = [rng.choice([0, 1, 2, 7, 64]) for _ in range(batch)]
    want = [0]
    for n in splits:
        want.append(want[-1] + n)
    assert chunk_prefix(splits) == want
    assert (batch + 31) // 32 <= MAX_COMPACT // 32   # the kernel's per-lane length arrays hold the chunks


@pytest.mark.parametrize("seed", range(6))
def test_one_split_per_sequence_uses_the_dense_walk(seed):
    """bps >= the table width: the dense walk is taken (no prefix scan) and,
    with no split past any sequence's end, visits exactly the real items."""
    rng = random.Random(200 + seed)
    batch = rng.choice([1, 17, 256, 512])
    lens = [rng.randint(1, 288) for _ in range(batch)]
    max_blocks = max(math.ceil(n / 64) for n in lens)
    bps = max_blocks + rng.randint(0, 2)
    total, _ = enumerate_items(lens, bps, max_blocks)
    assert total == batch * HKV
    total, ctas, processed, merges, arrivals = simulate(lens, bps, max_blocks, 148, seed)
    assert sorted(processed) == sorted((b, 0, h) for b in range(batch) for h in range(HKV))
    assert merges == []
