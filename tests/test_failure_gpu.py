"""Failure paths on the GPU, without a fault: a bounded wait is made to run
out (a barrier or an exchange word that nothing completes, with a 1 ms
limit), the kernel reports B2_DEV_TIMEOUT in the caller's error word and
returns, the host raises, and the same process then runs a normal step that
matches the oracle.  The reference's analogue is the watchdog around an NPU
run and the raise on a run that did not complete
(scripts/run_npu_timeout.ps1:1-19, experiments/npu_direct.py:110-114)."""
import ctypes

import pytest
import torch

from conftest import load_pkg
from oracle import lfm2_attention as orc
from test_kernels_gpu import build_batch, check_close, rand_qkv

pytestmark = pytest.mark.gpu
LIMIT_NS = 1_000_000   # 1 ms


def _lib():
    return load_pkg("_lib")


def _elapsed_ms(fn):
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end)


def test_decode_step_wait_runs_out(cuda):
    """B2_TEST_STALL: one consumer warp of the first CTA waits on a barrier
    that nothing completes.  With a 1 ms limit the launch ends within a few
    ms (not the 2 s default), the error word says B2_DEV_TIMEOUT, check()
    raises and clears the counters, and the next step is correct."""
    lib = _lib()
    attn = load_pkg("attention")
    lengths = [100, 300, 5, 64]
    cache, hist = build_batch(lengths, cuda, seed=31)
    w = orc.attention_weights(0)
    runner = attn.PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], len(lengths), 1024, blocks_per_split=1)
    raw = rand_qkv(len(lengths), 61)
    qkv = raw.to(cuda)
    past = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    kp, vp = cache.pool(0)

    def stalled():
        attn.decode_step(qkv, past, k_pool=kp, v_pool=vp, block_tables=cache.block_tables(), blocks_per_split=1,
                         out=runner.out[:len(lengths)], part_ml=runner.part_ml, part_o=runner.part_o,
                         counters=runner.counters, dev_err=runner.dev_err, gamma_q=runner.gamma_q,
                         gamma_k=runner.gamma_k, cos=runner.cos, sin=runner.sin,
                         mode=lib.B2_NORM_QK | lib.B2_ROPE_QK | lib.B2_STORE_KV | lib.B2_TEST_STALL)

    lib.set_wait_limits(LIMIT_NS, 0)
    try:
        ms = _elapsed_ms(stalled)
    finally:
        lib.set_wait_limits()
    assert lib.get_wait_limits() == (2_000_000_000, 5_000_000_000)
    assert int(runner.dev_err.item()) & lib.B2_DEV_TIMEOUT
    assert ms < 500, f"stalled step took {ms:.1f} ms: the 1 ms limit was not applied"
    with pytest.raises(RuntimeError, match="bounded device wait ran out"):
        runner.check()
    assert int(runner.dev_err.item()) == 0 and int(runner.counters.abs().sum().item()) == 0
    # the same step again, without the stall (it rewrites the same slots)
    out = runner.step(0, qkv, past, past + 1, cache.block_tables())
    torch.cuda.synchronize()
    runner.check()
    for i, n in enumerate(lengths):
        ctx, k_all, v_all, _ = orc.decode_step(raw[i], hist[i][0], hist[i][1], n, w["q_gamma"], w["k_gamma"])
        check_close(out[i], ctx, f"seq {i} after the timed-out step")
        kd, vd = cache.read_dense(0, i, n + 1)
        assert torch.equal(kd.cpu(), k_all) and torch.equal(vd.cpu(), v_all)
    assert int(runner.counters.abs().sum().item()) == 0


def test_exchange_poll_runs_out(cuda):
    """b2_exchange_merge at world 2 on one GPU: this rank's words go to both
    areas, but nothing writes the other rank's words.  With a 1 ms poll limit
    the kernel reports B2_DEV_TIMEOUT and leaves the context unwritten; then
    a world-1 merge on a zeroed area writes O / l."""
    lib = _lib()
    c = lib.load()
    batch = 3
    nbytes = c.b2_exchange_bytes(2, batch)
    assert nbytes > 0
    areas_t = [torch.zeros(nbytes // 4, dtype=torch.int32, device=cuda) for _ in range(2)]
    g = torch.Generator().manual_seed(5)
    state_ml = torch.stack([torch.randn(batch, 16, generator=g), torch.rand(batch, 16, generator=g) + 0.5], -1)
    state_o = torch.randn(batch, 16, 64, generator=g)
    state_ml, state_o = state_ml.to(cuda).contiguous(), state_o.to(cuda).contiguous()
    sentinel = torch.full((batch, 16, 64), 7.0, dtype=torch.bfloat16, device=cuda)
    out = sentinel.clone()
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    areas = (ctypes.c_void_p * 2)(areas_t[0].data_ptr(), areas_t[1].data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    args = (ctypes.c_void_p(state_ml.data_ptr()), ctypes.c_void_p(state_o.data_ptr()), batch)

    lib.set_wait_limits(0, LIMIT_NS)
    try:
        ms = _elapsed_ms(lambda: lib.check(
            c.b2_exchange_merge(*args, areas, 2, 0, ctypes.c_void_p(out.data_ptr()),
                                ctypes.c_void_p(err.data_ptr()), stream), "b2_exchange_merge"))
    finally:
        lib.set_wait_limits()
    assert int(err.item()) == lib.B2_DEV_TIMEOUT
    assert ms < 500, f"exchange took {ms:.1f} ms: the 1 ms poll limit was not applied"
    assert torch.equal(out, sentinel), "the context was written although the exchange timed out"
    # this rank's words did reach the "peer" area: slot 0, rank 0, tagged step 1
    words = areas_t[1].view(torch.int64).cpu()
    assert int((words >> 32).eq(1).sum().item()) == batch * 16 * 66
    # the GPU is usable: a world-1 merge (the area zeroed again)
    err.zero_()
    areas_t[0].zero_()
    one = (ctypes.c_void_p * 1)(areas_t[0].data_ptr())
    lib.check(c.b2_exchange_merge(*args, one, 1, 0, ctypes.c_void_p(out.data_ptr()),
                                  ctypes.c_void_p(err.data_ptr()), stream), "b2_exchange_merge")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want = (state_o / state_ml[..., 1:2]).to(torch.bfloat16)
    assert torch.equal(out, want)
