"""GPU parity: libb2attn.so kernels against the CPU oracle (reference semantics).

Tolerances: KV append bit-exact; attention context
max-abs <= 2e-2 and relative L2 error <= 1e-2 against the reference's
PyTorch BF16 path (sdpa), fp32 accumulation on the GPU.
"""
import numpy as np
import pytest
import torch

from conftest import load_pkg
from oracle import lfm2_attention as orc

pytestmark = pytest.mark.gpu

ATOL = 2e-2
RTOL = 1e-2


def _lib():
    return load_pkg("_lib")


def _attn():
    return load_pkg("attention")


def _cache_mod():
    return load_pkg("paged_cache")


def check_close(got: torch.Tensor, ref: torch.Tensor, what: str):
    got = got.float().cpu()
    ref = ref.float().cpu()
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    err = (got - ref).abs().max().item()
    rel = ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    assert err <= ATOL and rel <= RTOL, f"{what}: max-abs {err:.3e}, rel {rel:.3e}"


def ulp_diff(a: torch.Tensor, b: torch.Tensor) -> np.ndarray:
    """Distance in bf16 ulps between two bf16 tensors (sign-magnitude order)."""
    def key(t):
        u = orc.bits(t.cpu()).astype(np.int32)
        return np.where(u & 0x8000, 0x8000 - (u & 0x7FFF), 0x8000 + u)
    return np.abs(key(a) - key(b))


def build_batch(lengths, dev, seed=0, capacity=None, fill=float("nan"), num_blocks=None):
    """Paged cache holding seeded N(0,1) histories of the given lengths."""
    cm = _cache_mod()
    cap = capacity or (max(lengths) + 1)
    nb = num_blocks or sum(cm.blocks_for(cap) for _ in lengths) + 3
    cache = cm.PagedKVCache(nb, cap, device=dev, shuffle_seed=seed, fill=fill)
    hist = []
    for i, n in enumerate(lengths):
        cache.add_sequence(n)
        k, v = orc.past_cache(100 * seed + i, n)
        cache.write_dense(0, i, k[0], v[0])
        hist.append((k[0], v[0]))
    return cache, hist


def rand_qkv(batch, seed, scale=0.6):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(batch, 2048, generator=g) * scale).to(torch.bfloat16)


def test_library_loaded_from_tree():
    lib = _lib().load()
    assert lib.b2_version() >= 100
    assert str(_lib().LIB_PATH).endswith("ryzenai-npu-lab_b200/libb2attn.so")


@pytest.mark.parametrize("lengths", [[0], [0, 1, 63, 64, 65, 127, 128, 1000]])
def test_append_rope_bit_exact_given_normed(cuda, lengths):
    """RoPE + append of already-normalised q/k: bit-exact vs the oracle."""
    lib = _lib()
    cache, _ = build_batch(lengths, cuda, seed=1)
    b = len(lengths)
    w = orc.attention_weights(0)
    raw = rand_qkv(b, 11)
    q_raw, k_raw, v = orc.split_qkv(raw)
    qn = orc.rms_norm(q_raw, w["q_gamma"])
    kn = orc.rms_norm(k_raw, w["k_gamma"])
    qkv = torch.cat([qn.reshape(b, -1), kn.reshape(b, -1), v.reshape(b, -1)], dim=1)
    cos, sin = orc.rope_cos_sin(lengths)
    q_ref, k_ref = orc.norm_rope_qk(qn, kn, None, None, cos, sin, norm=False)
    rc, rs = load_pkg("rope").rope_table(2048, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    q_out = torch.empty(b, 16, 64, dtype=torch.bfloat16, device=cuda)
    kp, vp = cache.pool(0)
    _attn().append_rope(qkv.to(cuda), torch.tensor(lengths, dtype=torch.int32, device=cuda), q_out=q_out,
                        dev_err=err, mode=lib.B2_ROPE_QK | lib.B2_STORE_KV, cos=rc, sin=rs,
                        k_pool=kp, v_pool=vp, block_tables=cache.block_tables())
    torch.cuda.synchronize()
    assert err.item() == 0
    assert torch.equal(q_out.cpu(), q_ref)
    for i, n in enumerate(lengths):
        kd, vd = cache.read_dense(0, i, n + 1)
        assert torch.equal(kd[:, n].cpu(), k_ref[i]), f"k row {n} of seq {i}"
        assert torch.equal(vd[:, n].cpu(), v[i]), f"v row {n} of seq {i}"


def test_append_with_norm_matches_oracle(cuda):
    """RMSNorm + RoPE + append from raw projections: the rotated q and the
    appended k and v are bit-identical to the oracle (the kernel sums the
    squares in torch's CPU order), 128 sequences x 24 head vectors."""
    lib = _lib()
    lengths = list(range(0, 640, 5))
    cache, _ = build_batch(lengths, cuda, seed=2)
    b = len(lengths)
    w = orc.attention_weights(0)
    raw = rand_qkv(b, 12)
    q_raw, k_raw, v = orc.split_qkv(raw)
    cos, sin = orc.rope_cos_sin(lengths)
    q_ref, k_ref = orc.norm_rope_qk(q_raw, k_raw, w["q_gamma"], w["k_gamma"], cos, sin)
    rc, rs = load_pkg("rope").rope_table(1024, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    q_out = torch.empty(b, 16, 64, dtype=torch.bfloat16, device=cuda)
    kp, vp = cache.pool(0)
    _attn().append_rope(raw.to(cuda), torch.tensor(lengths, dtype=torch.int32, device=cuda), q_out=q_out,
                        dev_err=err, gamma_q=w["q_gamma"].to(cuda), gamma_k=w["k_gamma"].to(cuda),
                        cos=rc, sin=rs, k_pool=kp, v_pool=vp, block_tables=cache.block_tables())
    torch.cuda.synchronize()
    assert err.item() == 0
    k_got = torch.stack([cache.read_dense(0, i, n + 1)[0][:, n] for i, n in enumerate(lengths)])
    v_got = torch.stack([cache.read_dense(0, i, n + 1)[1][:, n] for i, n in enumerate(lengths)])
    assert torch.equal(v_got.cpu(), v)
    for got, ref, name in [(q_out, q_ref, "q"), (k_got, k_ref, "k")]:
        d = ulp_diff(got, ref)
        assert (d == 0).all(), f"{name}: {(d != 0).sum()} of {d.size} elements differ (max {d.max()} ulps)"


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "three_kernels"])
@pytest.mark.parametrize("bps", [1, 2, 3, 16, 40, 64])
def test_decode_ragged_vs_oracle(cuda, bps, fused):
    lengths = [1, 2, 63, 64, 65, 127, 128, 129, 1000, 4097]
    cache, hist = build_batch([n - 1 for n in lengths], cuda, seed=3)
    b = len(lengths)
    w = orc.attention_weights(0)
    raw = rand_qkv(b, 13)
    runner = _attn().PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], b, 8192, blocks_per_split=bps,
                                          fused=fused)
    past = torch.tensor([n - 1 for n in lengths], dtype=torch.int32, device=cuda)
    out = runner.step(0, raw.to(cuda), past, past + 1, cache.block_tables())
    torch.cuda.synchronize()
    runner.check()
    for i, n in enumerate(lengths):
        ctx, _, _, _ = orc.decode_step(raw[i], hist[i][0], hist[i][1], n - 1, w["q_gamma"], w["k_gamma"])
        check_close(out[i], ctx, f"seq {i} len {n} bps {bps}")


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "three_kernels"])
def test_bad_block_is_flagged_not_faulted(cuda, fused):
    lengths = [100, 200]
    cache, _ = build_batch(lengths, cuda, seed=4)
    w = orc.attention_weights(0)
    runner = _attn().PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], 2, 1024, blocks_per_split=2,
                                          fused=fused)
    tables = cache.block_tables()
    tables[1, 1] = cache.num_blocks + 5   # outside the pool
    past = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    runner.step(0, rand_qkv(2, 14).to(cuda), past, past + 1, tables)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="outside the pool"):
        runner.check()
    # the context is still usable afterwards
    tables = cache.block_tables()
    runner.step(0, rand_qkv(2, 14).to(cuda), past, past + 1, tables)
    torch.cuda.synchronize()
    runner.check()


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "three_kernels"])
def test_length_beyond_table_is_flagged(cuda, fused):
    cache, _ = build_batch([10], cuda, seed=5, capacity=64)
    w = orc.attention_weights(0)
    runner = _attn().PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], 1, 1024, blocks_per_split=1,
                                          fused=fused)
    past = torch.tensor([64], dtype=torch.int32, device=cuda)   # slot 64 is past the 1-block table
    runner.step(0, rand_qkv(1, 15).to(cuda), past, past + 1, cache.block_tables())
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="outside the block table"):
        runner.check()


def test_host_rejects_bad_arguments(cuda):
    attn = _attn()
    lib = _lib()
    cache, _ = build_batch([10], cuda, seed=6)
    kp, vp = cache.pool(0)
    q = torch.zeros(1, 16, 64, dtype=torch.bfloat16, device=cuda)
    ml = torch.empty(1, 1, 16, 2, device=cuda)
    po = torch.empty(1, 1, 16, 64, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    seq = torch.tensor([11], dtype=torch.int32, device=cuda)
    with pytest.raises(ValueError):
        attn.decode_attn(q.float(), kp, vp, cache.block_tables(), seq, blocks_per_split=1,
                         part_ml=ml, part_o=po, dev_err=err)
    with pytest.raises(lib.B2Error):
        attn.decode_attn(q, kp, vp, cache.block_tables(), seq, blocks_per_split=1,
                         part_ml=ml, part_o=po, dev_err=err, scale=-1.0)


@pytest.mark.parametrize("max_ctas", [1, 3, 0])
def test_fused_step_matches_three_kernels(cuda, max_ctas):
    """The fused persistent kernel against append + decode + combine: the
    appended pools and q are bit-identical (same norm/RoPE arithmetic), the
    contexts agree within the attention tolerance (the fused kernel's
    products run on the tensor cores with bf16 probabilities), whatever the
    number of CTAs sharing the work; the work counters are back to zero after
    every call."""
    lengths = [0, 5, 63, 64, 200, 1000, 3000, 64 * 20 - 1]
    b = len(lengths)
    w = orc.attention_weights(0)
    outs = []
    for fused in (False, True):
        cache, _ = build_batch(lengths, cuda, seed=8, capacity=64 * 50)
        runner = _attn().PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], b, 4096, blocks_per_split=4,
                                              fused=fused, max_ctas=max_ctas)
        past = torch.tensor(lengths, dtype=torch.int32, device=cuda)
        res = []
        for step in range(3):   # three consecutive decode steps
            o = runner.step(0, rand_qkv(b, 30 + step).to(cuda), past + step, past + step + 1, cache.block_tables())
            res.append(o.clone())
        torch.cuda.synchronize()
        runner.check()
        if fused:
            assert int(runner.counters.abs().sum().item()) == 0
        outs.append((res, runner.q.clone(), cache.k.clone(), cache.v.clone()))
    (r0, q0, k0, v0), (r1, q1, k1, v1) = outs
    for step, (a, c) in enumerate(zip(r0, r1)):
        check_close(c, a, f"step {step}")
    assert torch.equal(q0, q1)
    assert torch.equal(k0.nan_to_num(7.0), k1.nan_to_num(7.0))
    assert torch.equal(v0.nan_to_num(7.0), v1.nan_to_num(7.0))


@pytest.mark.parametrize("bps", [1, 3])
def test_fused_step_large_batch_dense_items(cuda, bps):
    """More than 512 sequences: the fused kernel enumerates the dense (split,
    sequence, head) space and skips splits past each sequence's end (a table
    20 blocks wide, histories of at most 5 blocks).  bps 1 gives 20 splits
    (merged by the combine kernel), bps 3 gives 7 (merged in the kernel).
    Against the three-kernel path, and the oracle on a few sequences."""
    g = torch.Generator().manual_seed(40 + bps)
    lengths = torch.randint(0, 300, (600,), generator=g).tolist()
    b = len(lengths)
    w = orc.attention_weights(0)
    raw = rand_qkv(b, 41)
    outs = []
    for fused in (False, True):
        cache, hist = build_batch(lengths, cuda, seed=9, capacity=64 * 20)
        runner = _attn().PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], b, 4096, blocks_per_split=bps,
                                              fused=fused)
        past = torch.tensor(lengths, dtype=torch.int32, device=cuda)
        out = runner.step(0, raw.to(cuda), past, past + 1, cache.block_tables()).clone()
        torch.cuda.synchronize()
        runner.check()
        if fused:
            assert int(runner.counters.abs().sum().item()) == 0
        outs.append(out)
    check_close(outs[1], outs[0], f"600 sequences, bps {bps}: fused vs three kernels")
    for i in (0, 1, 2, 299, 599):
        ctx, _, _, _ = orc.decode_step(raw[i], hist[i][0], hist[i][1], lengths[i], w["q_gamma"], w["k_gamma"])
        check_close(outs[1][i], ctx, f"seq {i} len {lengths[i] + 1} bps {bps}")


@pytest.mark.parametrize("state", [False, True], ids=["context", "state"])
@pytest.mark.parametrize("bps", [1, 8])
def test_fused_step_empty_sequences(cuda, bps, state):
    """Attention without the append (seq_lens given) where some sequences have
    nothing to attend: their context is zero, or their fp32 state (-1e30, 0,
    0); the others match the oracle's (m, l, o) over their first seq_lens
    tokens with q at position past_lens.  The table is 5 blocks wide: bps 8
    is one split per sequence (the dense walk of the work, no prefix scan),
    bps 1 five splits (the compact walk through the prefix scan)."""
    attn = _attn()
    rope = load_pkg("rope")
    w = orc.attention_weights(0)
    lengths = [0, 5, 0, 64, 300, 0, 1, 129] * 5
    b = len(lengths)
    cache, hist = build_batch(lengths, cuda, seed=12, capacity=320)
    assert cache.max_blocks == 5
    raw = rand_qkv(b, 77)
    past = torch.tensor([n + 3 for n in lengths], dtype=torch.int32, device=cuda)   # q's RoPE position
    seq = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    splits = attn.num_splits_for(cache.max_blocks, bps)
    kp, vp = cache.pool(0)
    cos, sin = rope.rope_table(400, device=cuda)
    out = torch.full((b, 16, 64), 7.0, dtype=torch.bfloat16, device=cuda)
    sml = torch.full((b, 16, 2), 7.0, device=cuda)
    so = torch.full((b, 16, 64), 7.0, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    counters = torch.zeros(2 + 8 * b, dtype=torch.int32, device=cuda)
    attn.decode_step(raw.to(cuda), past, k_pool=kp, v_pool=vp, block_tables=cache.block_tables(),
                     blocks_per_split=bps, out=None if state else out,
                     part_ml=torch.empty(b, splits, 16, 2, device=cuda),
                     part_o=torch.empty(b, splits, 16, 64, device=cuda), counters=counters, dev_err=err,
                     gamma_q=w["q_gamma"].to(cuda), gamma_k=w["k_gamma"].to(cuda), cos=cos, sin=sin,
                     seq_lens=seq, state_ml=sml if state else None, state_o=so if state else None,
                     mode=_lib().B2_NORM_QK | _lib().B2_ROPE_QK)
    torch.cuda.synchronize()
    assert err.item() == 0 and int(counters.abs().sum().item()) == 0
    for i, n in enumerate(lengths):
        q_raw, k_raw, _ = orc.split_qkv(raw[i:i + 1])
        c, s = orc.rope_cos_sin([n + 3])
        q, _ = orc.norm_rope_qk(q_raw, k_raw, w["q_gamma"], w["k_gamma"], c, s)
        m, l, o = orc.partial_state(q[0], hist[i][0], hist[i][1])
        if state:
            if n == 0:
                assert (sml[i, :, 0] == -1.0e30).all() and (sml[i, :, 1] == 0).all() and (so[i] == 0).all()
                continue
            # (m, l, o) equal the oracle's up to a common factor (the kernel's m is in log2 units)
            assert torch.isfinite(sml[i]).all() and (sml[i, :, 1] > 0).all()
            check_close(so[i].cpu() / sml[i, :, 1].cpu()[:, None], o / l[:, None], f"seq {i} len {n}: state")
        elif n == 0:
            assert (out[i] == 0).all(), f"seq {i}: empty context not zero"
        else:
            check_close(out[i], o / l[:, None], f"seq {i} len {n}")


def test_fused_multi_step_decode_vs_oracle(cuda):
    """Eight consecutive decode steps crossing a block edge, each attending
    over the tokens appended by the previous steps."""
    lengths = [60, 127, 2]
    cache, hist = build_batch(lengths, cuda, seed=9, capacity=200)
    b = len(lengths)
    w = orc.attention_weights(0)
    runner = _attn().PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], b, 4096, blocks_per_split=1)
    ks = [h[0] for h in hist]
    vs = [h[1] for h in hist]
    for step in range(8):
        raw = rand_qkv(b, 50 + step)
        past = torch.tensor([n + step for n in lengths], dtype=torch.int32, device=cuda)
        out = runner.step(0, raw.to(cuda), past, past + 1, cache.block_tables())
        torch.cuda.synchronize()
        runner.check()
        for i, n in enumerate(lengths):
            ctx, k_all, v_all, _ = orc.decode_step(raw[i], ks[i], vs[i], n + step, w["q_gamma"], w["k_gamma"])
            check_close(out[i], ctx, f"step {step} seq {i}")
            # the whole cache after the append is the oracle's, bit for bit;
            # the oracle carries its own history into the next step
            kd, vd = cache.read_dense(0, i, n + step + 1)
            assert torch.equal(kd.cpu(), k_all), f"step {step} seq {i}: k cache"
            assert torch.equal(vd.cpu(), v_all), f"step {step} seq {i}: v cache"
            ks[i], vs[i] = k_all, v_all


@pytest.mark.parametrize("total,cut", [(300, 128), (5000, 2048), (64, 64), (10, 64), (10, 0)])
def test_split_sequence_states_merge(cuda, total, cut):
    """One sequence split along the token axis as two GPUs would hold it,
    emulated on one GPU: the head part attends over its tokens only (seq_lens,
    RoPE at the global position through an offset table), the tail part also
    appends the new token; both return fp32 states that b2_combine merges."""
    attn = _attn()
    rope = load_pkg("rope")
    w = orc.attention_weights(0)
    k, v = orc.past_cache(91, total)
    k, v = k[0], v[0]
    raw = rand_qkv(1, 92)
    ctx_ref, _, _, _ = orc.decode_step(raw[0], k, v, total, w["q_gamma"], w["k_gamma"])
    cos, sin = rope.rope_table(total + 8, device=cuda)
    cm = _cache_mod()
    parts = [(0, min(cut, total), False), (min(cut, total), total, True)]
    states = []
    for lo, hi, tail in parts:
        n = hi - lo
        cache = cm.PagedKVCache(cm.blocks_for(n + 1) + 1, n + 1, device=cuda, fill=float("nan"))
        cache.add_sequence(n)
        if n:
            cache.write_dense(0, 0, k[:, lo:hi], v[:, lo:hi])
        kp, vp = cache.pool(0)
        past = torch.tensor([total - lo], dtype=torch.int32, device=cuda)
        seq = torch.tensor([n], dtype=torch.int32, device=cuda)
        splits = attn.num_splits_for(cache.max_blocks, 2)
        ml = torch.empty(1, splits, 16, 2, device=cuda)
        po = torch.empty(1, splits, 16, 64, device=cuda)
        sml = torch.empty(1, 16, 2, device=cuda)
        so = torch.empty(1, 16, 64, device=cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        mode = _lib().B2_NORM_QK | _lib().B2_ROPE_QK | (_lib().B2_STORE_KV if tail else 0)
        attn.decode_step(raw.to(cuda), past, k_pool=kp, v_pool=vp, block_tables=cache.block_tables(),
                         blocks_per_split=2, out=None, part_ml=ml, part_o=po,
                         counters=torch.zeros(2 + 8, dtype=torch.int32, device=cuda), dev_err=err,
                         gamma_q=w["q_gamma"].to(cuda), gamma_k=w["k_gamma"].to(cuda), cos=cos[lo:], sin=sin[lo:],
                         seq_lens=None if tail else seq, state_ml=sml, state_o=so, mode=mode)
        torch.cuda.synchronize()
        assert err.item() == 0
        states.append((sml, so))
    ml = torch.stack([s[0] for s in states], dim=1).contiguous()   # [1, 2, 16, 2]
    po = torch.stack([s[1] for s in states], dim=1).contiguous()   # [1, 2, 16, 64]
    out = torch.empty(1, 16, 64, dtype=torch.bfloat16, device=cuda)
    attn.combine(ml, po, 2, 1, out=out)
    # the same merge from the packed layout one all-gather produces
    packed = torch.stack([torch.cat([s[0].reshape(-1), s[1].reshape(-1)]) for s in states])
    out2 = torch.empty(1, 16, 64, dtype=torch.bfloat16, device=cuda)
    attn.merge_states(packed, 2, 1, out=out2)
    torch.cuda.synchronize()
    check_close(out[0], ctx_ref, f"split at {cut} of {total}")
    assert torch.equal(out, out2)


@pytest.mark.parametrize("double_buffered", [True, False])
def test_step_host_pipeline_matches_step(cuda, double_buffered):
    """The host-fed pipeline (pinned H2D, fused kernel, D2H; two device slots
    or one) returns what step() returns for the same inputs, over several steps."""
    lengths = [5, 300, 64, 1000]
    b = len(lengths)
    w = orc.attention_weights(0)
    outs = []
    keep = []   # pinned inputs stay alive until the stream is synchronised
    for host in (False, True):
        cache, _ = build_batch(lengths, cuda, seed=31, capacity=1100)
        runner = _attn().PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], b, 2048, blocks_per_split=4)
        tables = cache.block_tables()
        res = []
        if host:
            runner.open_host_pipeline(0, tables, double_buffered=double_buffered)
            out_host = torch.empty(5, b, 16, 64, dtype=torch.bfloat16).pin_memory()
        for step in range(5):
            raw = rand_qkv(b, 60 + step)
            past = torch.tensor([n + step for n in lengths], dtype=torch.int32)
            if host:
                keep.append((raw.pin_memory(), past.pin_memory()))
                runner.step_host(*keep[-1], out_host[step])
            else:
                res.append(runner.step(0, raw.to(cuda), past.to(cuda), (past + 1).to(cuda), tables).cpu())
        if host:
            runner.join_host()
        torch.cuda.synchronize()
        runner.check()
        outs.append(list(out_host) if host else res)
    for step, (a, c) in enumerate(zip(*outs)):
        assert torch.equal(a, c), f"step {step}"


def test_step_host_table_swap(cuda):
    """set_host_tables moves the host-fed pipeline between two block tables of
    one pool (the same histories in other blocks) from step to step: every
    step's context equals step() over the table it was given, and a table of
    another shape is refused."""
    lengths = [5, 300, 64]
    b = len(lengths)
    w = orc.attention_weights(0)
    outs = []
    keep = []
    for host in (False, True):
        cache, _ = build_batch(lengths + lengths, cuda, seed=37, capacity=400)
        for i, n in enumerate(lengths):   # copy 1 holds copy 0's histories in its own blocks
            k, v = orc.past_cache(100 * 37 + i, n)
            cache.write_dense(0, b + i, k[0], v[0])
        runner = _attn().PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], b, 1024, blocks_per_split=2)
        all_tables = cache.block_tables()
        tables = [all_tables[:b].contiguous(), all_tables[b:].contiguous()]
        res = []
        if host:
            runner.open_host_pipeline(0, tables[0])
            with pytest.raises(ValueError):
                runner.set_host_tables(all_tables)
            out_host = torch.empty(4, b, 16, 64, dtype=torch.bfloat16).pin_memory()
        for step in range(4):
            raw = rand_qkv(b, 80 + step)
            past = torch.tensor([n + step // 2 for n in lengths], dtype=torch.int32)
            if host:
                runner.set_host_tables(tables[step % 2])
                keep.append((raw.pin_memory(), past.pin_memory()))
                runner.step_host(*keep[-1], out_host[step])
            else:
                res.append(runner.step(0, raw.to(cuda), past.to(cuda), (past + 1).to(cuda), tables[step % 2]).cpu())
        if host:
            runner.join_host()
        torch.cuda.synchronize()
        runner.check()
        outs.append(list(out_host) if host else res)
    for step, (a, c) in enumerate(zip(*outs)):
        assert torch.equal(a, c), f"step {step}"
    assert not torch.equal(outs[0][0], outs[0][1])   # the two tables' steps saw different new tokens


def test_step_host_buffer_checks(cuda):
    """step_host refuses pageable or wrongly sized host buffers on every call,
    and accepts each row of one pinned buffer (its storage checked once):
    the same inputs give the same context in either row."""
    lengths = [5, 70]
    b = len(lengths)
    w = orc.attention_weights(0)
    cache, _ = build_batch(lengths, cuda, seed=33, capacity=200)
    runner = _attn().PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], b, 512, blocks_per_split=4)
    runner.open_host_pipeline(0, cache.block_tables())
    raw = rand_qkv(b, 7)
    qkv_h = raw.pin_memory()
    past_h = torch.tensor(lengths, dtype=torch.int32).pin_memory()
    out_h = torch.zeros(2, b, 16, 64, dtype=torch.bfloat16).pin_memory()
    with pytest.raises(ValueError):
        runner.step_host(raw.clone(), past_h, out_h[0])                        # pageable qkv
    with pytest.raises(ValueError):
        runner.step_host(qkv_h, past_h, torch.empty(b, 16, 64, dtype=torch.bfloat16))   # pageable out
    runner.step_host(qkv_h, past_h, out_h[0])
    with pytest.raises(ValueError):
        runner.step_host(qkv_h, past_h, out_h[1][:1])                          # a row short
    with pytest.raises(ValueError):
        runner.step_host(qkv_h, past_h.clone(), out_h[1])                      # pageable lengths
    runner.step_host(qkv_h, past_h, out_h[1])   # the same token again: the same slot, the same context
    runner.join_host()
    torch.cuda.synchronize()
    runner.check()
    assert torch.equal(out_h[0], out_h[1]) and out_h[0].abs().sum() > 0
