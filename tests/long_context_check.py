"""Long-context split-KV decode across the ranks of a torchrun job, checked
against the CPU oracle on every rank.  Run by tests/test_long_context_gpu.py:

    python -m torch.distributed.run --standalone --nproc-per-node N tests/long_context_check.py TOTAL EXCHANGE

Each rank holds a block-aligned token range of one sequence; every rank
computes a partial softmax state; the states are exchanged (EXCHANGE "p2p":
b2_exchange_merge over NVLink peer memory; "collective": NCCL all-gather +
merge kernel) and merged.  Five decode steps are run (the new token lives on
the last rank), so the exchange's two slots are each reused.
Exit status 0 when every step's context is within the attention tolerance.
"""
import datetime
import importlib
import os
import pathlib
import sys

import torch
import torch.distributed as dist

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
from oracle import lfm2_attention as orc  # noqa: E402

dmod = importlib.import_module("ryzenai-npu-lab_b200.distributed")


def main():
    total = int(sys.argv[1]) if len(sys.argv) > 1 else 5000
    exchange = sys.argv[2] if len(sys.argv) > 2 else "collective"
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    rank = dist.get_rank()
    w = orc.attention_weights(0)
    k, v = orc.past_cache(77, total)
    k, v = k[0], v[0]
    steps = 5
    lc = dmod.LongContextDecode(total + steps, w["q_gamma"], w["k_gamma"], device=dev, blocks_per_split=4,
                                growth=steps + 64, exchange=exchange)
    want = "direct" if dist.get_world_size() == 1 else exchange
    assert lc.exchange == want, (lc.exchange, want)
    lc.load_history(k, v)
    ok = True
    for step in range(steps):
        g = torch.Generator().manual_seed(500 + step)
        raw = (torch.randn(1, 2048, generator=g) * 0.6).to(torch.bfloat16)
        lc.set_lengths(total + step)
        out = lc.step(raw.to(dev))
        torch.cuda.synchronize()
        lc.check()
        ctx, k, v, _ = orc.decode_step(raw[0], k, v, total + step, w["q_gamma"], w["k_gamma"])
        # the oracle carries its own history (the GPU's appended rows are
        # bit-identical to it: tests/test_kernels_gpu.py)
        got = out.float().cpu()
        err = (got - ctx.float()).abs().max().item()
        rel = ((got - ctx.float()).norm() / ctx.float().norm()).item()
        print(f"rank {rank} step {step} ({lc.exchange}): max-abs {err:.3e} rel {rel:.3e}", flush=True)
        ok &= err <= 2e-2 and rel <= 1e-2 and bool(torch.isfinite(got).all())
    lc.close()
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    dist.destroy_process_group()
    sys.exit(int(flag.item() != 0))


if __name__ == "__main__":
    main()
