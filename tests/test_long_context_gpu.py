"""Long-context split-KV decode (config C4) over every visible GPU (up to 4,
one rank per GPU), as a torchrun subprocess: the partial states exchanged over
NVLink peer memory (b2_exchange_merge) or by an NCCL all-gather."""
import os
import pathlib
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = pathlib.Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("exchange", ["p2p", "collective"])
@pytest.mark.parametrize("total", [200, 5000])
def test_long_context_split_kv(cuda, total, exchange):
    n = min(torch.cuda.device_count(), 4)
    if exchange == "p2p" and n < 2:
        pytest.skip("the P2P exchange needs two GPUs (one rank per GPU)")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--local-addr", "127.0.0.1",
           "--nproc-per-node", str(n),
           str(ROOT / "tests" / "long_context_check.py"), str(total), exchange]
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
