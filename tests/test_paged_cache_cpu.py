"""The paged cache's host logic: block allocation, release and the block
tables the kernels read (CPU tensors; no kernel is launched)."""
import pytest
import torch

from conftest import load_pkg


def test_allocator_hands_out_each_block_once():
    pc = load_pkg("paged_cache")
    a = pc.BlockAllocator(16, shuffle_seed=5)
    got = a.alloc(10) + a.alloc(6)
    assert sorted(got) == list(range(16)) and a.free == 0
    with pytest.raises(MemoryError):
        a.alloc(1)
    a.release(got[:4])
    assert sorted(a.alloc(4)) == sorted(got[:4])


def test_allocator_refuses_bad_releases():
    pc = load_pkg("paged_cache")
    a = pc.BlockAllocator(8)
    got = a.alloc(3)
    with pytest.raises(ValueError, match="outside"):
        a.release([8])
    with pytest.raises(ValueError, match="not allocated"):
        a.release([got[0], 7])             # 7 was never handed out
    with pytest.raises(ValueError, match="twice"):
        a.release([got[0], got[0]])
    assert a.free == 5                     # refused releases release nothing
    a.release(got)
    with pytest.raises(ValueError, match="not allocated"):
        a.release([got[1]])                # double free
    assert a.free == 8 and sorted(a.alloc(8)) == list(range(8))


def test_release_sequence_returns_its_blocks():
    pc = load_pkg("paged_cache")
    cache = pc.PagedKVCache(num_blocks=6, capacity_tokens=128, device="cpu", shuffle_seed=1)
    s0, s1, s2 = cache.add_sequence(10), cache.add_sequence(70), cache.add_sequence(128)
    assert cache.allocator.free == 0
    with pytest.raises(MemoryError):
        cache.add_sequence(1)
    freed = cache.table(s1)
    cache.release_sequence(s1)
    t = cache.block_tables()
    assert t.shape == (3, 2) and t[s1].tolist() == [-1, -1] and cache.lengths[s1] == 0
    s3 = cache.add_sequence(5)
    assert sorted(cache.table(s3)) == sorted(freed)
    cache.release_sequence(s1)             # a released row holds no blocks: nothing happens,
    assert cache.allocator.free == 0       # and s3's blocks (once s1's) stay allocated
    assert sorted(cache.table(s0) + cache.table(s2) + cache.table(s3)) == list(range(6))


@pytest.mark.parametrize("lengths", [[1, 63, 64, 65, 200], [0, 129, 7]])
def test_pool_layout_the_kernels_index(lengths):
    """Token t of sequence s, KV head h sits at pool[table[s][t // 64], h, t % 64, :]
    (the [block][8][64][64] layout every kernel's tensor map and append
    address assume), and read_dense returns exactly what write_dense stored,
    across block boundaries and with shuffled blocks; other sequences' blocks
    are untouched."""
    pc = load_pkg("paged_cache")
    cap = max(lengths) + 1
    cache = pc.PagedKVCache(num_blocks=sum(pc.blocks_for(cap) for _ in lengths) + 2, capacity_tokens=cap,
                            num_layers=2, device="cpu", shuffle_seed=11, fill=0.0)
    g = torch.Generator().manual_seed(3)
    hist = []
    for s, n in enumerate(lengths):
        assert cache.add_sequence(n) == s
        k = torch.randn(8, n, 64, generator=g).to(torch.bfloat16)
        v = torch.randn(8, n, 64, generator=g).to(torch.bfloat16)
        cache.write_dense(1, s, k, v)
        hist.append((k, v))
    kp, vp = cache.pool(1)
    tables = cache.block_tables()
    assert tables.dtype == torch.int32 and tables.shape == (len(lengths), pc.blocks_for(cap))
    for s, (n, (k, v)) in enumerate(zip(lengths, hist)):
        for t in {0, n // 2, n - 1} if n else set():
            blk = int(tables[s, t // 64])
            for h in (0, 5, 7):
                assert torch.equal(kp[blk, h, t % 64], k[h, t]) and torch.equal(vp[blk, h, t % 64], v[h, t])
        rk, rv = cache.read_dense(1, s, n)
        assert torch.equal(rk, k) and torch.equal(rv, v)
    assert cache.pool(0)[0].abs().sum() == 0      # the other layer's pool was not written
    used = {int(b) for b in tables.flatten() if b >= 0}
    assert len(used) == sum(pc.blocks_for(cap) for _ in lengths)
    free_ids = sorted(set(range(cache.num_blocks)) - used)
    assert kp[free_ids].abs().sum() == 0          # nor the blocks no sequence holds
