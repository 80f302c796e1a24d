"""Host-side multi-GPU logic on CPU: sequence sharding, token ranges, and the
long-context state exchange over a world-size-2 gloo group (the partial
states come from the CPU oracle; on GPUs they come from libb2attn.so)."""
import ctypes
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_pkg
from oracle import lfm2_attention as orc


def test_shard_sequences_balances_tokens():
    dist_mod = load_pkg("distributed")
    g = torch.Generator().manual_seed(3)
    lengths = torch.randint(128, 8193, (64,), generator=g).tolist()
    for world in (1, 2, 4, 8):
        shards = dist_mod.shard_sequences(lengths, world)
        assert sorted(i for s in shards for i in s) == list(range(64))
        loads = [sum(lengths[i] + 1 for i in s) for s in shards]
        assert max(loads) - min(loads) <= max(lengths) + 1
    with pytest.raises(ValueError):
        dist_mod.shard_sequences(lengths, 0)


@pytest.mark.parametrize("total", [0, 1, 63, 64, 65, 1000, 131072, 131073])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_token_ranges_cover_and_align(total, world):
    dist_mod = load_pkg("distributed")
    r = dist_mod.token_ranges(total, world)
    assert len(r) == world
    assert r[0][0] == 0 and r[-1][1] == total
    for (a, b), (c, _) in zip(r, r[1:]):
        assert b == c and a <= b
    for a, b in r:
        assert a % 64 == 0 or a == b == total   # empty trailing ranges sit at the end
    sizes = [b - a for a, b in r]
    assert max(sizes) - min(sizes) <= 64 * 2


def test_p2p_exchange_needs_one_host_and_distinct_gpus():
    dist_mod = load_pkg("distributed")
    assert dist_mod.p2p_possible(["h", "h"], ["GPU-a", "GPU-b"])
    assert not dist_mod.p2p_possible(["h", "h"], ["GPU-a", "GPU-a"])     # two ranks on one GPU
    assert not dist_mod.p2p_possible(["h", "g"], ["GPU-a", "GPU-b"])     # two hosts
    assert not dist_mod.p2p_possible(["h"], ["GPU-a"])                   # a world of one merges directly
    assert not dist_mod.p2p_possible(["h"] * 9, [f"GPU-{i}" for i in range(9)])


def test_exchange_area_size():
    lib = load_pkg("_lib").load()
    # [2 slots][world][batch][16][68] tagged 8-byte words + [batch][16] step counters
    assert lib.b2_exchange_bytes(2, 1) == 2 * 2 * 16 * 68 * 8 + 16 * 4
    assert lib.b2_exchange_bytes(8, 3) == 2 * 8 * 3 * 16 * 68 * 8 + 3 * 16 * 4
    assert lib.b2_exchange_bytes(9, 1) == 0 and lib.b2_exchange_bytes(0, 1) == 0 and lib.b2_exchange_bytes(2, 0) == 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _long_context_worker(rank, world, port, total, q, k, v, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dist_mod = load_pkg("distributed")
        lo, hi = dist_mod.token_ranges(total, world)[rank]
        m, l, o = orc.partial_state(q, k[:, lo:hi], v[:, lo:hi])
        state = torch.cat([m[:, None], l[:, None], o], dim=1)[None]      # [1, 16, 66]
        allst = dist_mod.gather_states(state)                              # [world, 1, 16, 66]
        parts = [(s[0, :, 0], s[0, :, 1], s[0, :, 2:]) for s in allst]
        result[rank] = orc.merge_states(parts)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("total", [300, 1000])
def test_long_context_state_exchange_gloo(total):
    world = 2
    g = torch.Generator().manual_seed(11)
    q = torch.randn(16, 64, generator=g).to(torch.bfloat16)
    k = torch.randn(8, total, 64, generator=g).to(torch.bfloat16)
    v = torch.randn(8, total, 64, generator=g).to(torch.bfloat16)
    full = orc.attend(q[None, :, None, :], k[None], v[None], "fp32").reshape(16, 64)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_long_context_worker, args=(r, world, port, total, q, k, v, result))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        for r in range(world):
            assert torch.allclose(result[r], full, atol=1e-5, rtol=1e-5)


def _exchange_choice_worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dist_mod = load_pkg("distributed")
        g = torch.ones(64, dtype=torch.bfloat16)
        lc = dist_mod.LongContextDecode(1000, g, g, device="cpu", growth=64)
        out = [lc.exchange, lc.start, lc.end, lc.is_tail]
        for bad in ("p2p", "bogus"):
            try:
                dist_mod.LongContextDecode(1000, g, g, device="cpu", growth=64, exchange=bad)
                out.append("accepted")
            except ValueError:
                out.append("ValueError")
        result[rank] = out
    finally:
        dist.destroy_process_group()


def test_long_context_exchange_choice_gloo():
    """On CPU ranks (gloo) the exchange falls back to the collective; asking
    for the P2P kernel, or an unknown exchange, is a ValueError."""
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_exchange_choice_worker, args=(r, world, port, result)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        assert result[0] == ["collective", 0, 512, False, "ValueError", "ValueError"]
        assert result[1] == ["collective", 512, 1000, True, "ValueError", "ValueError"]


def test_split_size_heuristic():
    attn = load_pkg("attention")
    # one long sequence: ~2 equal items per SM in one wave (8 KV heads x splits <= 296)
    for blocks in (2049, 1026, 514, 258):
        bps = attn.choose_blocks_per_split(1, blocks, fused=True)
        splits = -(-blocks // bps)
        assert 1 <= bps <= 64 and splits * 8 <= 2 * 148
    assert attn.choose_blocks_per_split(1, 4097, fused=True) == 64      # capped: several equal waves
    # many sequences: ~6 items per resident CTA, 4..32 blocks
    assert attn.choose_blocks_per_split(64, 3715, fused=True) == 12
    # the 64-sequence batch sharded over 2/4/8 GPUs (longest 129 blocks): the
    # measured best split sizes; at 32 sequences at most 16 splits (merged in
    # the kernel) with ~3 items per resident CTA
    for batch, work, want in ((32, 1860, 9), (16, 930, 6), (8, 470, 6)):
        assert attn.choose_blocks_per_split(batch, work, fused=True, max_blocks_per_seq=129) == want
    assert 4 <= attn.choose_blocks_per_split(512, 512 * 60, fused=True) <= 32
    # three-kernel path: ~8 CTAs of work per SM
    assert 2 <= attn.choose_blocks_per_split(64, 3715) <= 64


def _open_peers_worker(rank, world, port, fail_on, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dist_mod = load_pkg("distributed")
        closed = []

        def open_fn(entry):
            if (rank, entry) == fail_on:
                raise RuntimeError("b2_ipc_open failed")
            return 1000 + entry

        def close_fn(ptr, entry):
            closed.append(ptr)

        entries = list(range(world))      # rank r's "handle" is r
        try:
            opened, ptrs = dist_mod.open_peer_areas(entries, rank, open_fn, close_fn)
            out = ["ok", [p for p, _ in opened], ptrs]
        except ValueError as e:
            out = ["ValueError", str(e)]
        dist.barrier()                     # every rank reaches the next collective
        result[rank] = out + [sorted(closed)]
    finally:
        dist.destroy_process_group()


def _run_open_peers(world, fail_on):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_open_peers_worker, args=(r, world, port, fail_on, result))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        return dict(result)


def test_peer_setup_agrees_on_failure_gloo():
    """One rank that cannot map a peer's area makes every rank raise ValueError
    (so an automatic choice falls back to the collective on all of them), and
    the ranks that did map areas unmap them."""
    res = _run_open_peers(3, fail_on=(1, 2))
    for r in range(3):
        assert res[r][0] == "ValueError" and "rank 1: mapping rank 2's area" in res[r][1]
    assert res[0][2] == [1001, 1002]       # rank 0 mapped ranks 1 and 2, then unmapped both
    assert res[1][2] == [1000]             # rank 1 mapped rank 0 before failing on rank 2
    assert res[2][2] == [1000, 1001]


def test_peer_setup_success_gloo():
    res = _run_open_peers(2, fail_on=None)
    assert res[0] == ["ok", [1001], [None, 1001], []]
    assert res[1] == ["ok", [1000], [1000, None], []]


class _FakeIpcLib:
    """Stands in for libb2attn.so's exchange entry points on CPU ranks."""

    def __init__(self, rank, fail_handle):
        self.rank, self.fail_handle, self.closed = rank, fail_handle, []

    def b2_exchange_bytes(self, world, batch):
        return 256

    def b2_ipc_handle(self, ptr, handle, offset_ref):
        if self.fail_handle:
            return -2
        ctypes.memmove(handle, b"rank%d" % self.rank, 5)
        offset_ref._obj.value = 16 * (self.rank + 1)
        return 0

    def b2_ipc_open(self, handle, offset, peer_ref):
        peer_ref._obj.value = 4096 * (int(handle[4:5]) + 1) + offset
        return 0

    def b2_ipc_close(self, ptr, offset):
        self.closed.append((ptr.value, offset))
        return 0


def _peer_exchange_worker(rank, world, port, fail_handle_rank, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lib_mod = load_pkg("_lib")
        dist_mod = load_pkg("distributed")
        fake = _FakeIpcLib(rank, rank == fail_handle_rank)
        lib_mod.load = lambda: fake
        lib_mod.last_error = lambda: "fake failure"
        torch.cuda.get_device_properties = lambda dev: type("P", (), {"uuid": f"GPU-{rank}"})()
        torch.cuda.synchronize = lambda dev=None: None
        try:
            px = dist_mod.PeerExchange(1, device="cpu")
            areas = list(px.areas)
            areas[rank] = "own" if areas[rank] == px.area.data_ptr() else areas[rank]
            px.close()
            result[rank] = ["ok", areas, fake.closed]
        except ValueError as e:
            dist.barrier()
            result[rank] = ["ValueError", str(e)]
    finally:
        dist.destroy_process_group()


def _run_peer_exchange(world, fail_handle_rank):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_peer_exchange_worker, args=(r, world, port, fail_handle_rank, result))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        return dict(result)


def test_peer_exchange_setup_and_close_gloo():
    """PeerExchange's host logic with a fake IPC library: every rank maps the
    others' areas from the gathered handles and offsets, and close() unmaps
    exactly those."""
    res = _run_peer_exchange(3, fail_handle_rank=None)
    for r in range(3):
        status, areas, closed = res[r]
        assert status == "ok" and areas[r] == "own"
        peers = [(4096 * (p + 1) + 16 * (p + 1), 16 * (p + 1)) for p in range(3) if p != r]
        assert [a for i, a in enumerate(areas) if i != r] == [a for a, _ in peers]
        assert sorted(closed) == sorted(peers)


def test_peer_exchange_handle_failure_is_everyones_gloo():
    res = _run_peer_exchange(2, fail_handle_rank=1)
    for r in range(2):
        assert res[r][0] == "ValueError" and "rank 1: b2_ipc_handle: fake failure" in res[r][1]


def _device_error_worker(rank, world, port, words, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lib_mod = load_pkg("_lib")
        dist_mod = load_pkg("distributed")
        failed = dist_mod.agree_device_errors(words[rank])
        out = ["raised" if failed else "clean", failed]
        if failed:
            # the recovery every rank then runs together: PeerExchange.reset()
            # (fake IPC library; the barriers must pair up on every rank)
            fake = _FakeIpcLib(rank, False)
            lib_mod.load = lambda: fake
            torch.cuda.get_device_properties = lambda dev: type("P", (), {"uuid": f"GPU-{rank}"})()
            torch.cuda.synchronize = lambda dev=None: None
            px = dist_mod.PeerExchange(1, device="cpu")
            px.area.fill_(7)
            px.reset()
            out.append(int(px.area.abs().sum()))
            px.close()
        dist.barrier()
        result[rank] = out
    finally:
        dist.destroy_process_group()


def test_device_errors_agreed_by_every_rank_gloo():
    """A bounded wait that ran out on one rank only (its dev_err word set, the
    other's clear): every rank learns of it and raises, then all reset the
    exchange areas together without waiting for one another in vain."""
    lib = load_pkg("_lib")
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        words = [0, lib.B2_DEV_TIMEOUT]
        procs = [ctx.Process(target=_device_error_worker, args=(r, 2, port, words, result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        res = dict(result)
    for r in range(2):
        assert res[r][0] == "raised", res
        assert res[r][1] == ["rank 1: a bounded device wait ran out"], res
        assert res[r][2] == 0      # the area is zero after reset()


def test_device_errors_clean_on_every_rank_gloo():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_device_error_worker, args=(r, 2, port, [0, 0], result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        res = dict(result)
    assert res[0] == ["clean", []] and res[1] == ["clean", []]
