"""bench.py's contract pieces that run without a GPU: the reference arm's JSON
line (timed on the host cores) and the per-rank workload of the scaling runs."""
import json
import subprocess
import sys
import types

from conftest import ROOT


def test_reference_arm_prints_one_json_line():
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2",
                           "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert "workload" in d["config"]
    assert d["cpu_baseline"]["mean_context"] == d["config"]["context_mean"]
    # the same config dict the GPU arm prints for the same flags (one function of the job's lengths)
    sys.path.insert(0, str(ROOT))
    import bench
    argv = sys.argv
    try:
        sys.argv = ["bench.py", "--impl", "reference", "--steps", "2", "--warmup", "1"]
        args = bench.parse()
    finally:
        sys.argv = argv
    assert d["config"] == bench.config_block(args, bench.base_lengths(args), 1)


def test_small_shards_rotate_over_copies_larger_than_l2():
    """Every rank of the strong-scaling runs streams at least twice L2 of K/V
    between two reads of the same block: N = 1 reads its 0.49 GB once per
    step, N = 2 / 4 / 8 ranks rotate over 2 / 3 / 5 copies of their share."""
    sys.path.insert(0, str(ROOT))
    import bench
    a = types.SimpleNamespace(seed=3, min_len=128, max_len=8192, batch=64, scaling="strong")   # bench's default draw
    want = {1: 1, 2: 2, 4: 3, 8: 5}
    for world in (1, 2, 4, 8):
        for rank in range(world):
            lengths = bench.seq_lengths(a, rank, world)
            footprint, copies = bench.rotation_copies(lengths)
            assert footprint == sum(2048 * (n + 1) for n in lengths)
            assert copies * footprint >= 2 * bench.L2_BYTES
            assert copies == 1 or (copies - 1) * footprint < 2 * bench.L2_BYTES
            assert copies == want[world], (world, rank, copies)
    assert bench.rotation_copies([])[1] >= 1


def test_strong_scaling_shards_the_one_batch():
    """Default (strong): the one seeded 64-sequence batch is split over the
    ranks, 64/32/16/8 per GPU, every sequence on exactly one rank, balanced
    by cached tokens."""
    sys.path.insert(0, str(ROOT))
    import bench
    a = types.SimpleNamespace(seed=3, min_len=128, max_len=8192, batch=64, scaling="strong")
    base = sorted(bench.seq_lengths(a, 0, 1))
    assert len(base) == 64
    for world in (2, 4, 8):
        shards = [bench.seq_lengths(a, rank, world) for rank in range(world)]
        assert sorted(sum(shards, [])) == base
        assert all(len(sh) == 64 // world for sh in shards)
        tokens = [sum(sh) for sh in shards]
        assert max(tokens) - min(tokens) <= max(base)
        assert bench.global_tokens_per_step(a, world) == 64


def test_weak_scaling_gives_every_rank_the_one_gpu_batch():
    sys.path.insert(0, str(ROOT))
    import bench
    a = types.SimpleNamespace(seed=3, min_len=128, max_len=8192, batch=64, scaling="weak")
    base = sorted(bench.seq_lengths(a, 0, 1))
    for world in (2, 4, 8):
        for rank in range(world):
            assert sorted(bench.seq_lengths(a, rank, world)) == base
        assert bench.global_tokens_per_step(a, world) == 64 * world


def test_cpu_baseline_sample_is_the_whole_workload():
    """The CPU baseline loops over all 64 sequences, so its mean context is
    the workload's (not a longer or shorter subset)."""
    sys.path.insert(0, str(ROOT))
    import bench
    a = types.SimpleNamespace(seed=3, min_len=128, max_len=8192, batch=64, scaling="strong")
    lengths = bench.base_lengths(a)
    rate, info = bench.cpu_reference_rate(lengths, 0.0)
    assert rate > 0 and info["sequences"] == 64
    assert info["mean_context"] == round(sum(lengths) / 64, 1)
    assert bench.config_block(types.SimpleNamespace(**vars(a), gpus=1), lengths, 1)["context_mean"] == \
        info["mean_context"]


def test_reference_arm_other_ranks_exit_quietly():
    """Under torchrun with N > 1 only rank 0 runs the reference arm; rank 1
    prints nothing and exits 0 (its environment is what torchrun sets)."""
    import os
    env = dict(os.environ, RANK="1", LOCAL_RANK="1", WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
               MASTER_PORT="29599")
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2",
                           "--steps", "2", "--warmup", "1"], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert proc.stdout.strip() == ""


def test_algorithmic_bytes_follow_the_formula():
    """bytes per step = sum over sequences of 2048 (L + 4) + 4 ceil((L + 1) / 64):
    K and V of L cached tokens, the raw q/k/v read, the k/v append, the
    context write, and the block-table entries."""
    sys.path.insert(0, str(ROOT))
    import bench
    step, decode = bench.step_bytes([0, 63, 64])
    assert step == (2048 * 4 + 4) + (2048 * 67 + 4) + (2048 * 68 + 8)
    assert decode == (2048 * 1 + 2048 + 4) + (2048 * 64 + 2048 + 4) + (2048 * 65 + 2048 + 8)
    a = types.SimpleNamespace(seed=3, min_len=128, max_len=8192, batch=64, scaling="strong")
    step, _ = bench.step_bytes(bench.seq_lengths(a, 0, 1))
    assert 0.45e9 < step < 0.65e9          # ~546 MB per layer-step for 64 sequences of mean ~4 K
