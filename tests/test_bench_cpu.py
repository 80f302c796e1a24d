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


def test_every_rank_gets_the_one_gpu_batch():
    sys.path.insert(0, str(ROOT))
    import bench
    a = types.SimpleNamespace(seed=3, min_len=128, max_len=8192, batch=64)
    base = sorted(bench.seq_lengths(a, 0, 1))
    assert len(base) == 64
    for world in (2, 4, 8):
        for rank in range(world):
            assert sorted(bench.seq_lengths(a, rank, world)) == base


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
    a = types.SimpleNamespace(seed=3, min_len=128, max_len=8192, batch=64)
    step, _ = bench.step_bytes(bench.seq_lengths(a, 0, 1))
    assert 0.45e9 < step < 0.65e9          # ~546 MB per layer-step for 64 sequences of mean ~4 K
