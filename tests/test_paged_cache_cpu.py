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
