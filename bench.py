"""Benchmark of the LFM2.5 decode-attention hot path on B200.

    python bench.py --gpus N --steps K --warmup W [--impl b200|reference]

Workload (batched paged decode): 64 sequences with
cached lengths uniform in [128, 8192] (one seeded draw), K/V ~ N(0, 1) bf16 in
a pool of 64-token blocks handed out in shuffled order, 16 q heads / 8 KV
heads / head_dim 64.  One step = one decode token per sequence through one
attention layer: fused q/k RMSNorm + RoPE + KV append, split-KV flash-decode,
combine.  With N GPUs the 64 sequences are sharded over the GPUs by token
count (64/32/16/8 per GPU at 1/2/4/8; strong scaling, the default) with no
collective; `--scaling weak` gives every GPU its own copy of the 64-sequence
batch instead.  The step time is the max over ranks.  The K/V pool (~0.49 GB)
is larger than L2 (126 MB), so no L2 flush is needed between steps.

At N = 1 the line also carries `contexts`: fixed-length batches of 32 and 64
sequences at 1K/4K/8K/16K cached tokens (the metric's "vs context" axis) and
config C2 (one sequence, 6 layers x 64 steps) from 1K/4K/16K.  Points whose
K/V would fit in L2 rotate over enough copies of the batch (separate block
tables in one pool) that every step reads memory the previous steps did not.

The timed region replays a CUDA graph of exactly K steps with inputs already
in HBM; `e2e` times the same steps through the public API
(PagedDecodeAttention.step_host, one b2_decode_step_host2 call per step) with
the per-step inputs copied from pinned host memory and the context copied
back inside the timed region (uploads and downloads overlap the neighbouring
steps' kernels).

`--impl reference` times the reference's CPU path (the oracle's restatement
of transformers' Lfm2Attention + DynamicCache in BF16) on this host's cores,
on bounded samples of the same workload.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import pathlib
import statistics
import sys
import threading
import time

import torch

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
PKG = "ryzenai-npu-lab_b200"
METRIC = "decode-attn tokens/s & HBM GB/s (% of 8 TB/s) vs context at 1/2/4/8 B200"
HQ, HKV, D, BLOCK = 16, 8, 64, 64
KV_BYTES_PER_TOKEN = 2 * HKV * D * 2          # K + V, bf16: 2048 B
L2_BYTES = 126 * 2 ** 20
FALLBACK_HBM_GBS = 6650.0


def parse():
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=400)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--batch", type=int, default=64, help="sequences per GPU")
    p.add_argument("--min-len", type=int, default=128)
    p.add_argument("--max-len", type=int, default=8192)
    p.add_argument("--bps", type=int, default=0, help="blocks per split (0 = heuristic)")
    p.add_argument("--seed", type=int, default=3)
    p.add_argument("--e2e-steps", type=int, default=100)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="bounded CPU baseline sample")
    p.add_argument("--three-kernels", action="store_true",
                   help="run append, decode and combine as three launches instead of the fused kernel")
    p.add_argument("--max-ctas", type=int, default=0, help="cap on the fused kernel's persistent grid")
    p.add_argument("--chunk", type=int, default=64, help="prefill: new tokens per sequence")
    p.add_argument("--prefill-bps", type=int, default=-1,
                   help="prefill: blocks per key split (-1 = heuristic, 0 = no split)")
    p.add_argument("--prefill-kernel", choices=["tcgen05", "step"], default="tcgen05",
                   help="prefill: tcgen05 = the batched prompt kernel; step = the fused decode step for "
                        "chunks of up to 4 tokens (b2_decode_step_tokens)")
    p.add_argument("--config", choices=["c3", "c4", "c1", "c2", "c5", "prefill"], default="c3",
                   help="c3: batched paged decode (default); c4: one long sequence split over the GPUs; "
                        "c1: one attention layer (projections included) for one token at 512 cached tokens; "
                        "c2: 6 attention layers x 64 consecutive decode steps of one sequence; "
                        "c5: end-to-end greedy decode of the whole random-init model; "
                        "prefill: a chunk of --chunk new tokens per C3 sequence on the tcgen05 kernel")
    p.add_argument("--context", type=int, default=131072, help="c4: cached tokens of the sequence")
    p.add_argument("--torch-glue", action="store_true",
                   help="c5: run the layer glue (norms, SwiGLU, short conv) as torch ops")
    p.add_argument("--b2-gemm", action="store_true",
                   help="c5: the layer projections on b2_gemm (tcgen05) instead of cuBLAS")
    p.add_argument("--exchange", choices=["auto", "p2p", "collective"], default="auto",
                   help="c4: how the ranks' partial states are merged")
    p.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                   help="c3 with N GPUs: shard the one 64-sequence batch (strong) or give every GPU a copy (weak)")
    p.add_argument("--no-sweep", action="store_true", help="c3: skip the vs-context points")
    p.add_argument("--shard", type=str, default="",
                   help="c3 on one GPU: run only rank R's shard of an N-GPU job, given as R/N "
                        "(its sequences and work, to study one rank of the scaling runs)")
    return p.parse_args()


# ----------------------------------------------------------------- helpers

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_hbm_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic_per_kv_token(kernel: str):
    """DRAM bytes per cached token of `kernel` from its committed ncu summary
    (profiles/<kernel>_c3.txt, line 'traffic_bytes_per_kv_token: X')."""
    path = ROOT / "profiles" / f"{kernel}_c3.txt"
    try:
        for line in path.read_text().splitlines():
            if line.startswith("traffic_bytes_per_kv_token:"):
                return float(line.split(":")[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index: int, period: float = 0.002):
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._period = period
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nvml.nvmlDeviceGetClockInfo(self._h, self._nvml.NVML_CLOCK_SM))
                self.reasons |= self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self._nvml is not None:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._nvml is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0}
        names = [n for n, bit in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# ----------------------------------------------------------------- workload

def base_lengths(args) -> list[int]:
    """The C3 batch: one seeded draw of --batch cached lengths."""
    g = torch.Generator().manual_seed(args.seed * 1000)
    return torch.randint(args.min_len, args.max_len + 1, (args.batch,), generator=g).tolist()


def seq_lengths(args, rank: int, world: int = 1) -> list[int]:
    """Cached lengths of this rank's sequences.  Strong scaling (default): the
    one C3 batch sharded over the ranks by token count (longest first to the
    least-loaded rank), 64/32/16/8 sequences per GPU at 1/2/4/8.  Weak: the
    global batch is N copies of it (different K/V per rank), so every GPU gets
    exactly the work of the one-GPU run."""
    base = base_lengths(args)
    if world == 1:
        return base
    lengths = base * world if getattr(args, "scaling", "strong") == "weak" else base
    dmod = importlib.import_module(PKG + ".distributed")
    return [lengths[i] for i in dmod.shard_sequences(lengths, world)[rank]]


def global_tokens_per_step(args, world: int) -> int:
    """Decode tokens the whole job produces per step (one per sequence)."""
    return args.batch * (world if getattr(args, "scaling", "strong") == "weak" else 1)


def synthetic_attention_weights(seed: int, hidden: int = 1024) -> dict:
    """Seeded random-init weights of one LFM2.5 attention layer (the configs'
    N(0, 0.02) projections; q/k RMSNorm gains 1 + N(0, 0.1)), bf16 on the host."""
    g = torch.Generator().manual_seed(seed)
    w = {"q_proj": torch.randn(HQ * D, hidden, generator=g) * 0.02,
         "k_proj": torch.randn(HKV * D, hidden, generator=g) * 0.02,
         "v_proj": torch.randn(HKV * D, hidden, generator=g) * 0.02,
         "out_proj": torch.randn(hidden, HQ * D, generator=g) * 0.02,
         "q_gamma": 1.0 + 0.1 * torch.randn(D, generator=g),
         "k_gamma": 1.0 + 0.1 * torch.randn(D, generator=g)}
    return {k: v.to(torch.bfloat16) for k, v in w.items()}


def synthetic_lfm2_weights(seed: int, dev, hidden: int = 1024, ffn: int = 2560, vocab: int = 65536) -> dict:
    """Seeded random-init LFM2.5-230M-shaped weights under Hugging Face
    parameter names, drawn on the device: matrices N(0, 0.02), short-conv taps
    N(0, 0.3), norm gains 1 (q/k layernorm gains 1 + N(0, 0.1)), the head tied
    to the embedding; the layer pattern is the runner's (8 short-conv, 6 GQA)."""
    runner_mod = importlib.import_module(PKG + ".lfm2_runner")
    g = torch.Generator(device=dev).manual_seed(seed)

    def n(*shape, std=0.02):
        return (torch.randn(*shape, generator=g, device=dev) * std).to(torch.bfloat16)

    def ones(k):
        return torch.ones(k, dtype=torch.bfloat16, device=dev)

    sd = {"model.embed_tokens.weight": n(vocab, hidden)}
    for i, kind in enumerate(runner_mod.LFM25_LAYER_TYPES):
        p = f"model.layers.{i}."
        if kind == "attention":
            sd[p + "self_attn.q_proj.weight"] = n(HQ * D, hidden)
            sd[p + "self_attn.k_proj.weight"] = n(HKV * D, hidden)
            sd[p + "self_attn.v_proj.weight"] = n(HKV * D, hidden)
            sd[p + "self_attn.out_proj.weight"] = n(hidden, HQ * D)
            sd[p + "self_attn.q_layernorm.weight"] = (1.0 + n(D, std=0.1).float()).to(torch.bfloat16)
            sd[p + "self_attn.k_layernorm.weight"] = (1.0 + n(D, std=0.1).float()).to(torch.bfloat16)
        else:
            sd[p + "conv.conv.weight"] = n(hidden, 1, 3, std=0.3)
            sd[p + "conv.in_proj.weight"] = n(3 * hidden, hidden)
            sd[p + "conv.out_proj.weight"] = n(hidden, hidden)
        sd[p + "feed_forward.w1.weight"] = n(ffn, hidden)
        sd[p + "feed_forward.w3.weight"] = n(ffn, hidden)
        sd[p + "feed_forward.w2.weight"] = n(hidden, ffn)
        sd[p + "operator_norm.weight"] = ones(hidden)
        sd[p + "ffn_norm.weight"] = ones(hidden)
    sd["model.embedding_norm.weight"] = ones(hidden)
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    return sd


def rotation_copies(lengths) -> tuple[int, int]:
    """(K/V bytes one step reads, copies of the sequences its steps rotate
    over).  A shard whose K/V would stay in L2 from one step to the next (4 or
    8 ranks of the strong-scaling batch) is held `copies` times in its own
    blocks and the steps rotate over the copies' block tables, so that the
    K/V streamed between two reads of a block is at least twice L2."""
    footprint = sum(KV_BYTES_PER_TOKEN * (n + 1) for n in lengths)
    return footprint, max(1, math.ceil(2 * L2_BYTES / max(1, footprint)))


def build_workload(args, rank: int, dev: torch.device, world: int = 1):
    attn = importlib.import_module(PKG + ".attention")
    pc = importlib.import_module(PKG + ".paged_cache")
    lengths = seq_lengths(args, rank, world)
    caps = [n + 1 for n in lengths]
    footprint, copies = rotation_copies(lengths)
    num_blocks = copies * sum(pc.blocks_for(c) for c in caps)
    cache = pc.PagedKVCache(num_blocks, max(caps), device=dev, shuffle_seed=args.seed * 1000 + rank + 17)
    for _ in range(copies):
        for n, c in zip(lengths, caps):
            cache.add_sequence(n, capacity=c)
    gen = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank + 29)
    cache.k.normal_(generator=gen)
    cache.v.normal_(generator=gen)
    gg = torch.Generator().manual_seed(args.seed * 1000 + rank + 31)
    gamma_q = (1.0 + 0.1 * torch.randn(D, generator=gg)).to(torch.bfloat16)
    gamma_k = (1.0 + 0.1 * torch.randn(D, generator=gg)).to(torch.bfloat16)
    work_blocks = sum(pc.blocks_for(c) for c in caps)
    runner = attn.PagedDecodeAttention(cache, gamma_q, gamma_k, len(lengths), args.max_len + 2,
                                       blocks_per_split=args.bps or None, work_blocks=work_blocks,
                                       fused=not args.three_kernels, max_ctas=args.max_ctas)
    ring = 8
    qkv = (torch.randn(ring, len(lengths), 2048, generator=gen, device=dev) * 0.6).to(torch.bfloat16)
    past = torch.tensor(lengths, dtype=torch.int32, device=dev)
    nb = len(lengths)
    all_tables = cache.block_tables()
    tables = [all_tables[c * nb:(c + 1) * nb].contiguous() for c in range(copies)]
    return {"lengths": lengths, "cache": cache, "runner": runner, "qkv": qkv, "past": past,
            "seq": past + 1, "tables": tables[0], "table_ring": tables, "copies": copies,
            "kv_bytes": footprint, "ring": ring}


def step_bytes(lengths) -> tuple[int, int]:
    """Algorithmic HBM bytes: (whole step, decode kernel) for one step."""
    nblk = [math.ceil((n + 1) / BLOCK) for n in lengths]
    step = sum(KV_BYTES_PER_TOKEN * (n + 4) + 4 * b for n, b in zip(lengths, nblk))
    decode = sum(KV_BYTES_PER_TOKEN * (n + 1) + HQ * D * 2 + 4 * b for n, b in zip(lengths, nblk))
    return step, decode


# ----------------------------------------------------------------- CPU reference path

def cpu_reference_rate(lengths, seconds: float, seed: int = 0):
    """tokens/s of the reference CPU path (oracle restatement of transformers'
    Lfm2Attention decode + DynamicCache.update) over sequences of the given
    lengths, one sequence at a time (the reference decode loop is batch-1),
    with all host threads.  Every sequence of `lengths` takes part, so the
    sample's mean context is the workload's; runs whole passes over them until
    `seconds` have elapsed (at least one pass)."""
    from oracle import lfm2_attention as orc

    torch.set_num_threads(os.cpu_count() or 1)
    w = orc.attention_weights(seed)
    g = torch.Generator().manual_seed(seed + 1)
    sample = list(lengths)
    hist = [(torch.randn(HKV, n, D, generator=g).to(torch.bfloat16),
             torch.randn(HKV, n, D, generator=g).to(torch.bfloat16)) for n in sample]
    qkv = (torch.randn(len(sample), 2048, generator=g) * 0.6).to(torch.bfloat16)
    cos, sin = orc.rope_cos_sin(sample)
    # warm-up
    orc.decode_step(qkv[0], hist[0][0], hist[0][1], sample[0], w["q_gamma"], w["k_gamma"],
                    cos=cos[0:1], sin=sin[0:1])
    done, t0 = 0, time.perf_counter()
    while True:
        for i, n in enumerate(sample):
            orc.decode_step(qkv[i], hist[i][0], hist[i][1], n, w["q_gamma"], w["k_gamma"],
                            cos=cos[i:i + 1], sin=sin[i:i + 1])
            done += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return done / el, {"sequences": len(sample), "seq_steps": done, "seconds": round(el, 2),
                       "mean_context": round(sum(sample) / len(sample), 1)}


def cpu_sample_info(info: dict) -> str:
    return (f"batch-1 loop over all {info['sequences']} sequences of the workload (mean context "
            f"{info['mean_context']}), {info['seq_steps']} sequence-steps in {info['seconds']} s")


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    lengths = base_lengths(args)
    per_step = max(0.02, min(1.0, 60.0 / max(1, args.steps)))   # whole run ~1 min
    for _ in range(args.warmup):
        cpu_reference_rate(lengths[:4], 0.0)
    rates, info = [], None
    for _ in range(args.steps):
        r, info = cpu_reference_rate(lengths, per_step)
        rates.append(r)
    value = statistics.median(rates)
    cores = torch.get_num_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * args.batch / value, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_block(args, lengths, args.gpus),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"median of {args.steps} samples, each a {cpu_sample_info(info)}",
                         "mean_context": info["mean_context"]},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def l2_policy(lengths, world: int, weak: bool) -> str:
    """How the steps avoid reading K/V out of L2 (build_workload), from the
    job's lengths alone, so that both arms print the same config."""
    total = sum(KV_BYTES_PER_TOKEN * (n + 1) for n in lengths) * (world if weak else 1)
    per_rank = total / world
    return (f"{total / 1e6:.0f} MB of K/V per step over {world} GPU(s), ~{per_rank / 1e6:.0f} MB per rank; "
            f"a rank whose share is under 2x L2 (126 MB) rotates its steps over copies of its sequences "
            f"in their own blocks, so every step streams its K/V from HBM; no flush")


def config_block(args, lengths, world: int = 1):
    """lengths: every sequence of the job (all ranks)."""
    weak = args.scaling == "weak" and world > 1
    return {
        "workload": f"C3 batched paged decode: {args.batch} sequences, cached length ~U[{args.min_len}, "
                    f"{args.max_len}], 64-token bf16 KV blocks in shuffled order, 16q/8kv heads x 64; one step = "
                    "one decode token per sequence through one attention layer "
                    "(q/k norm + RoPE + KV append, split-KV flash-decode, combine); "
                    + (f"every GPU decodes its own copy of the batch (weak scaling)" if weak else
                       f"the sequences sharded over {world} GPU(s) by token count (strong scaling)"),
        "global_batch": global_tokens_per_step(args, world), "batch_per_gpu": "sharded" if not weak else args.batch,
        "context_min": args.min_len, "context_max": args.max_len,
        "context_mean": round(sum(lengths) / len(lengths), 1),
        "block_tokens": BLOCK, "parallelism": f"seq-shard x{world}",
        "l2": l2_policy(base_lengths(args), world, weak),
    }


# ----------------------------------------------------------------- vs-context points



def time_graph(graph, stream, reps: int = 1) -> float:
    """ms of `reps` replays of a captured graph, CUDA events on its stream."""
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        t0.record()
        for _ in range(reps):
            graph.replay()
        t1.record()
    torch.cuda.synchronize()
    return t0.elapsed_time(t1)


def fixed_batch_point(args, dev, batch: int, L: int, steps: int = 96) -> dict:
    """One decode step of `batch` sequences that all hold L cached tokens,
    through the fused kernel (the C3 step at a fixed context).  If the K/V of
    the batch would stay in L2, the step rotates over `copies` batches with
    their own blocks (at least 4x L2 in all), so every step streams from HBM."""
    attn = importlib.import_module(PKG + ".attention")
    pc = importlib.import_module(PKG + ".paged_cache")
    cap = L + 1
    footprint = batch * KV_BYTES_PER_TOKEN * cap
    copies = max(1, math.ceil(4 * L2_BYTES / footprint))
    cache = pc.PagedKVCache(batch * copies * pc.blocks_for(cap), cap, device=dev,
                            shuffle_seed=args.seed * 1000 + L + batch)
    for _ in range(batch * copies):
        cache.add_sequence(L, capacity=cap)
    gen = torch.Generator(device=dev).manual_seed(args.seed * 1000 + L + batch + 29)
    cache.k.normal_(generator=gen)
    cache.v.normal_(generator=gen)
    gg = torch.Generator().manual_seed(args.seed + 31)
    gq = (1.0 + 0.1 * torch.randn(D, generator=gg)).to(torch.bfloat16)
    gk = (1.0 + 0.1 * torch.randn(D, generator=gg)).to(torch.bfloat16)
    runner = attn.PagedDecodeAttention(cache, gq, gk, batch, cap + 1, work_blocks=batch * pc.blocks_for(cap))
    all_tables = cache.block_tables()
    tables = [all_tables[c * batch:(c + 1) * batch].contiguous() for c in range(copies)]
    ring = 4
    qkv = (torch.randn(ring, batch, 2048, generator=gen, device=dev) * 0.6).to(torch.bfloat16)
    past = torch.full((batch,), L, dtype=torch.int32, device=dev)
    seq = past + 1
    steps = copies * math.ceil(steps / copies)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for j in range(max(3, copies)):
            runner.step(0, qkv[j % ring], past, seq, tables[j % copies])
    stream.synchronize()
    runner.check()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for j in range(steps):
            runner.step(0, qkv[j % ring], past, seq, tables[j % copies])
    time_graph(graph, stream)   # upload
    ms = time_graph(graph, stream) / steps
    runner.check()
    nbytes = batch * (KV_BYTES_PER_TOKEN * (L + 4) + 4 * pc.blocks_for(cap))
    peak, _ = measured_hbm_peak()
    gbs = nbytes / (ms / 1e3) / 1e9
    del graph, runner, cache
    torch.cuda.empty_cache()
    return {"batch": batch, "context": L, "us_per_step": round(1e3 * ms, 2),
            "tokens_per_s": round(batch / (ms / 1e3), 1), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
            "pct_of_8tbs": round(100 * gbs / 8000, 2), "copies": copies, "steps": steps}


def c2_point(args, dev, L0: int, reps: int = 4, sampler=None) -> dict:
    """Config C2 from L0 cached tokens: one sequence, 6 attention layers x 64
    consecutive decode steps (each appends one token per layer), captured once
    as a CUDA graph and replayed; per token = 6 fused steps."""
    attn = importlib.import_module(PKG + ".attention")
    pc = importlib.import_module(PKG + ".paged_cache")
    layers, steps = 6, 64
    cap = L0 + steps + 1
    cache = pc.PagedKVCache(pc.blocks_for(cap), cap, num_layers=layers, device=dev,
                            shuffle_seed=args.seed * 1000 + 17)
    cache.add_sequence(L0, capacity=cap)
    gen = torch.Generator(device=dev).manual_seed(args.seed * 1000 + 29)
    cache.k.normal_(generator=gen)
    cache.v.normal_(generator=gen)
    gg = torch.Generator().manual_seed(args.seed + 31)
    gammas = [((1.0 + 0.1 * torch.randn(D, generator=gg)).to(torch.bfloat16),
               (1.0 + 0.1 * torch.randn(D, generator=gg)).to(torch.bfloat16)) for _ in range(layers)]
    runners = [attn.PagedDecodeAttention(cache, gq, gk, 1, cap + 1, blocks_per_split=args.bps or None,
                                         work_blocks=pc.blocks_for(cap)) for gq, gk in gammas]
    qkv = (torch.randn(steps, layers, 1, 2048, generator=gen, device=dev) * 0.6).to(torch.bfloat16)
    past = torch.arange(L0, L0 + steps, dtype=torch.int32, device=dev).reshape(steps, 1)
    seq = past + 1
    tables = cache.block_tables()
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for t in range(3):
            for layer in range(layers):
                runners[layer].step(layer, qkv[t, layer], past[t], seq[t], tables)
    stream.synchronize()
    for r in runners:
        r.check()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for t in range(steps):
            for layer in range(layers):
                runners[layer].step(layer, qkv[t, layer], past[t], seq[t], tables)
    time_graph(graph, stream)   # upload
    if sampler is not None:
        with sampler:
            ms = time_graph(graph, stream, reps) / (reps * steps)
    else:
        ms = time_graph(graph, stream, reps) / (reps * steps)
    for r in runners:
        r.check()
    nbytes = sum(layers * (KV_BYTES_PER_TOKEN * (L0 + t + 4) + 4 * pc.blocks_for(L0 + t + 1))
                 for t in range(steps)) / steps
    peak, _ = measured_hbm_peak()
    gbs = nbytes / (ms / 1e3) / 1e9
    out = {"context": L0, "layers": layers, "us_per_token": round(1e3 * ms, 2),
           "tokens_per_s": round(1 / (ms / 1e3), 1), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
           "blocks_per_split": runners[0].blocks_per_split, "splits": runners[0].num_splits}
    del graph, runners, cache
    torch.cuda.empty_cache()
    return out


def guarded(fn, *a, **kw):
    """An extra point of the N = 1 line: its failure is recorded in the line
    rather than costing the headline measurement."""
    try:
        return fn(*a, **kw)
    except Exception as e:   # noqa: BLE001 - reported in the JSON line
        return {"error": f"{type(e).__name__}: {e}"[:400]}


def context_sweep(args, dev) -> dict:
    """The metric's 'vs context' axis on one GPU (after the headline run)."""
    points = [fixed_batch_point(args, dev, b, L) for b in (32, 64) for L in (1024, 4096, 8192, 16384)]
    return {"note": "fused decode step, one token per sequence and layer, all sequences at the given "
                    "context; frac of the measured HBM copy peak; copies > 1: the step rotates over that "
                    "many batches so that its K/V is not served from L2",
            "batched": points,
            "c2": [c2_point(args, dev, L0) for L0 in (1024, 4096, 16384)],
            # config C4 on one GPU: one sequence of 131 072 cached tokens (the step splits its keys
            # over the CTAs and merges them with the combine kernel)
            "c4_one_gpu": guarded(fixed_batch_point, args, dev, 1, 131072, steps=48)}


# ----------------------------------------------------------------- B200 path

def run_b200(args):
    world, rank, local = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py: no CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
        pg = torch.distributed.group.WORLD
    if args.shard:
        if world != 1:
            raise SystemExit("--shard runs one rank's shard in a single process")
        srank, sworld = (int(x) for x in args.shard.split("/"))
        wl = build_workload(args, srank, dev, sworld)
    else:
        wl = build_workload(args, rank, dev, world)
    runner = wl["runner"]
    K, W, ring = args.steps, args.warmup, wl["ring"]
    stream = torch.cuda.Stream(dev)
    torch.cuda.synchronize()

    def one_step(j, ev=None):
        runner.step(0, wl["qkv"][j % ring], wl["past"], wl["seq"], wl["tables"])

    # warm-up (untimed) also sets up the kernels' attributes before capture
    with torch.cuda.stream(stream):
        for j in range(max(W, 1)):
            one_step(j)
    stream.synchronize()
    runner.check()

    # CUDA graph of exactly K steps.  The fused kernel is the whole step, so
    # its launch time is the timed region / K (no event nodes between the
    # launches); with three kernels, external events bracket the decode launch.
    attn = importlib.import_module(PKG + ".attention")
    ev0 = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(K)]
    ev1 = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(K)]
    graph = torch.cuda.CUDAGraph()
    kp, vp = runner.cache.pool(0)
    b = len(wl["lengths"])
    copies = wl["copies"]
    with torch.cuda.graph(graph, stream=stream):
        for j in range(K):
            tables = wl["table_ring"][j % copies]
            if runner.fused:
                runner.step(0, wl["qkv"][j % ring], wl["past"], wl["seq"], tables)
                continue
            q = runner.q[:b]
            attn.append_rope(wl["qkv"][j % ring], wl["past"], q_out=q, dev_err=runner.dev_err,
                             gamma_q=runner.gamma_q, gamma_k=runner.gamma_k, cos=runner.cos, sin=runner.sin,
                             k_pool=kp, v_pool=vp, block_tables=tables)
            ev0[j].record()
            splits = attn.decode_attn(q, kp, vp, tables, wl["seq"],
                                      blocks_per_split=runner.blocks_per_split, part_ml=runner.part_ml,
                                      part_o=runner.part_o, dev_err=runner.dev_err)
            ev1[j].record()
            attn.combine(runner.part_ml, runner.part_o, splits, b, seq_lens=wl["seq"],
                         blocks_per_split=runner.blocks_per_split, out=runner.out[:b])
    graph.replay()   # one untimed replay (graph upload)
    torch.cuda.synchronize()
    runner.check()

    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    if pg is not None:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            t_start.record()
            graph.replay()
            t_end.record()
        torch.cuda.synchronize()
    if pg is not None:
        torch.distributed.barrier()
    ms = t_start.elapsed_time(t_end)
    decode_ms = ms / K if runner.fused else sum(a.elapsed_time(b) for a, b in zip(ev0, ev1)) / K
    runner.check()

    # end-to-end through the public API: pinned host inputs in, context out, per step
    e2e_steps = min(args.e2e_steps, K)
    qkv_host = wl["qkv"].cpu().pin_memory()
    past_host = wl["past"].cpu().pin_memory()
    nb = len(wl["lengths"])
    out_host = torch.empty(e2e_steps, nb, HQ, D, dtype=torch.bfloat16).pin_memory()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if runner.fused:
        # host-fed pipeline: per step H2D (copy stream), fused kernel, D2H
        with torch.cuda.stream(stream):
            runner.open_host_pipeline(0, wl["tables"])
            for j in range(3):
                runner.step_host(qkv_host[j % ring], past_host, out_host[j % e2e_steps])
            runner.join_host()
        torch.cuda.synchronize()
        if pg is not None:
            torch.distributed.barrier()
        with torch.cuda.stream(stream):
            e0.record()
            for j in range(e2e_steps):
                if copies > 1:
                    runner.set_host_tables(wl["table_ring"][j % copies])
                runner.step_host(qkv_host[j % ring], past_host, out_host[j])
            runner.join_host()
            e1.record()
    else:
        qkv_dev = torch.empty_like(wl["qkv"][0])
        lens_dev = torch.empty(2, nb, dtype=torch.int32, device=dev)
        lens_host = torch.stack([wl["past"].cpu(), wl["seq"].cpu()]).pin_memory()
        with torch.cuda.stream(stream):
            for j in range(3):
                qkv_dev.copy_(qkv_host[j % ring], non_blocking=True)
                runner.step(0, qkv_dev, wl["past"], wl["seq"], wl["tables"])
        torch.cuda.synchronize()
        if pg is not None:
            torch.distributed.barrier()
        with torch.cuda.stream(stream):
            e0.record()
            for j in range(e2e_steps):
                qkv_dev.copy_(qkv_host[j % ring], non_blocking=True)
                lens_dev.copy_(lens_host, non_blocking=True)
                o = runner.step(0, qkv_dev, lens_dev[0], lens_dev[1], wl["table_ring"][j % copies])
                out_host[j].copy_(o, non_blocking=True)
            e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    runner.check()

    ms_local = ms
    times = torch.tensor([ms, decode_ms, e2e_ms], dtype=torch.float64, device=dev)
    if pg is not None:
        torch.distributed.all_reduce(times, op=torch.distributed.ReduceOp.MAX)
    ms, decode_ms, e2e_ms = times.tolist()

    lengths = wl["lengths"]
    sbytes, dbytes = step_bytes(lengths)
    kernel = "paged_decode_kernel"
    if runner.fused:
        dbytes, kernel = sbytes, "decode_step_kernel"
    # every rank's own step time, sequences and cached tokens (which rank is the slow one)
    per_rank = torch.empty(world, 3, dtype=torch.float64, device=dev)
    mine = torch.tensor([[1e3 * ms_local / K, len(lengths), sum(lengths)]], dtype=torch.float64, device=dev)
    if pg is not None:
        torch.distributed.all_gather_into_tensor(per_rank, mine)
    else:
        per_rank.copy_(mine)
    per_rank_rows = [[round(r[0], 2), int(r[1]), int(r[2])] for r in per_rank.tolist()]
    peak, peak_kind = measured_hbm_peak()
    ms_step = ms / K
    tokens = global_tokens_per_step(args, world)
    value = tokens * K / (ms / 1e3)
    achieved = dbytes / (decode_ms / 1e3) / 1e9
    tpt = profiled_traffic_per_kv_token(kernel)
    kv_tokens = sum(n + 1 for n in lengths)
    step_gbs = sbytes / (ms_step / 1e3) / 1e9
    all_lengths = base_lengths(args) * (world if args.scaling == "weak" else 1)
    if args.shard:
        tokens = len(lengths)   # only this shard's sequences were decoded
        value = tokens * K / (ms / 1e3)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms_step, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_block(args, all_lengths, world),
        # this rank's kernel plan: work-item size, and how many copies of its
        # sequences the steps rotate over (1 = its K/V alone exceeds 2x L2)
        "plan": {"blocks_per_split": runner.blocks_per_split, "copies": copies,
                 "kv_mb_per_step": round(wl["kv_bytes"] / 1e6, 1)},
        "per_rank": {"columns": ["step_us", "sequences", "cached_tokens"], "rows": per_rank_rows},
        "hbm_gbs_per_gpu": step_gbs, "hbm_pct_of_8tbs": 100.0 * step_gbs / 8000.0,
        "roofline": {"bound": "hbm", "kernel": kernel, "achieved": achieved,
                     "peak": peak, "peak_source": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None if tpt is None else tpt * kv_tokens,
                     "algorithmic_bytes": dbytes, "avg_launch_ms": decode_ms},
        "clocks": clocks.summary(),
        "e2e": {"value": tokens * e2e_steps / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": nb * (2048 * 2 + (4 if runner.fused else 8)),
                "d2h_bytes_per_step": nb * HQ * D * 2, "steps": e2e_steps},
        # the fused step, plus the combine kernel when a sequence has more than 16 splits
        "gpu_launches": ((1 + (runner.num_splits > 16)) if runner.fused else 3) * K,
    }
    if args.shard:
        line["config"]["shard"] = args.shard
        line["config"]["workload"] += f"; ONLY shard {args.shard} of it on this GPU (one rank's part)"
        line["config"]["l2"] = l2_policy(base_lengths(args), int(args.shard.split("/")[1]),
                                         args.scaling == "weak")
    if rank == 0 and world == 1 and not args.no_sweep and not args.shard:
        line["contexts"] = context_sweep(args, dev)
        line["prefill"] = prefill_points(args, dev)
        # config C5 on this GPU (the default runner: cuBLAS projections, layer glue in libb2attn)
        c5 = guarded(c5_point, args, dev)
        if "ms" in c5:
            c5 = {"workload": "C5 end-to-end greedy decode, LFM2.5-230M-shaped random-init model, 256 prompts "
                              "x 32 ids, 256 new tokens (prefill included), paged KV, CUDA graph per token",
                  **{k: (round(v, 2) if isinstance(v, float) else v) for k, v in c5.items()}}
        line["c5"] = c5
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.shard:
        rate, info = cpu_reference_rate(base_lengths(args), args.cpu_seconds)
        line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": torch.get_num_threads(),
                                "kind": "port", "sample": "reference CPU path (transformers Lfm2Attention "
                                f"restated, DynamicCache cat + sdpa), {cpu_sample_info(info)}",
                                "mean_context": info["mean_context"]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    if pg is not None:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_c4(args):
    """Config C4: one sequence of --context cached tokens split along the token
    axis over the ranks; per step each rank appends (last rank) and attends over
    its tokens, the partial states are exchanged (NVLink P2P kernel, or an NCCL
    all-gather with --exchange collective) and merged."""
    import datetime
    world, rank, local = dist_env()
    if "RANK" not in os.environ:   # single process without torchrun: a world of one
        import socket
        with socket.socket() as sock:
            sock.bind(("127.0.0.1", 0))
            port = sock.getsockname()[1]
        os.environ.update(RANK="0", WORLD_SIZE="1", LOCAL_RANK="0", MASTER_ADDR="127.0.0.1",
                          MASTER_PORT=str(port))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    torch.distributed.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    dmod = importlib.import_module(PKG + ".distributed")
    K, W = args.steps, args.warmup
    gg = torch.Generator().manual_seed(args.seed + 31)
    gamma_q = (1.0 + 0.1 * torch.randn(D, generator=gg)).to(torch.bfloat16)
    gamma_k = (1.0 + 0.1 * torch.randn(D, generator=gg)).to(torch.bfloat16)
    lc = dmod.LongContextDecode(args.context + 1, gamma_q, gamma_k, device=dev,
                                blocks_per_split=args.bps or None, growth=64, exchange=args.exchange,
                                max_ctas=args.max_ctas)
    gen = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank + 29)
    lc.fill_random(args.context, gen)
    lc.set_lengths(args.context)
    qkv = (torch.randn(8, 1, 2048, generator=gen, device=dev) * 0.6).to(torch.bfloat16)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for j in range(max(W, 1)):
            lc.step(qkv[j % 8])
    stream.synchronize()
    lc.check()
    # the timed graph: K whole steps, no event nodes between the launches
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for j in range(K):
            lc.step(qkv[j % 8])
    # a second graph brackets the local partial of every step with events
    # (the roofline's kernel time); with one GPU the partial is the step
    ev0 = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(K)]
    ev1 = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(K)]
    graph_ev = None
    if world > 1:
        graph_ev = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_ev, stream=stream):
            for j in range(K):
                ev0[j].record()
                lc.partial(qkv[j % 8])
                ev1[j].record()
                lc.merge()
        graph_ev.replay()
    graph.replay()
    torch.cuda.synchronize()
    lc.check()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            # pre-roll: the ranks leave the host barrier milliseconds apart, and
            # the per-step exchange makes the early ones wait for the late ones;
            # one untimed replay brings them into step, then K steps are timed
            if world > 1:
                graph.replay()
            t0.record()
            graph.replay()
            t1.record()
        torch.cuda.synchronize()
    torch.distributed.barrier()
    lc.check()
    ms = t0.elapsed_time(t1)
    if graph_ev is not None:
        with torch.cuda.stream(stream):
            graph_ev.replay()
        torch.cuda.synchronize()
        lc.check()
        part_ms = sum(a.elapsed_time(b) for a, b in zip(ev0, ev1)) / K
    else:
        part_ms = ms / K
    local_tokens = lc.local_len + (1 if lc.is_tail else 0)
    local_bytes = KV_BYTES_PER_TOKEN * local_tokens + 2048 * 2 + 2 * 1024
    # every rank's own step time, partial time and tokens (which rank is the slow one), then the max
    per_rank = torch.empty(world, 3, dtype=torch.float64, device=dev)
    torch.distributed.all_gather_into_tensor(
        per_rank, torch.tensor([[1e3 * ms / K, 1e3 * part_ms, local_tokens]], dtype=torch.float64, device=dev))
    per_rank_rows = [[round(r[0], 2), round(r[1], 2), int(r[2])] for r in per_rank.tolist()]
    times = torch.tensor([ms, part_ms], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(times, op=torch.distributed.ReduceOp.MAX)
    ms, part_ms = times.tolist()
    peak, peak_kind = measured_hbm_peak()
    total_bytes = KV_BYTES_PER_TOKEN * (args.context + 1) + 2048 * 2 + 2 * 1024
    line = {
        "metric": METRIC, "value": K / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"C4 long-context decode: one sequence of {args.context} cached tokens "
                               f"split along the token axis over {world} GPU(s), partial softmax states "
                               + {"p2p": "merged by the combine kernel, which exchanges them with the other "
                                         "ranks over NVLink peer memory and merges the world's "
                                         "(b2_decode_step_exchange)",
                                  "collective": "all-gathered over NCCL and merged",
                                  "direct": "(one GPU: merged in the step)"}[lc.exchange],
                   "context": args.context, "exchange": lc.exchange,
                   "global_batch": 1, "blocks_per_split": lc.bps, "parallelism": f"split-kv x{world}",
                   "timing": "K steps after one untimed replay of the K-step graph (ranks in step)" if world > 1
                   else "K steps",
                   "l2": (f"{KV_BYTES_PER_TOKEN * args.context / 1e6:.0f} MB of K/V, "
                          f"~{KV_BYTES_PER_TOKEN * args.context / world / 1e6:.0f} MB per rank, no flush"
                          + ("; a rank's share fits in L2 (126 MB): its K/V loads carry an evict-first "
                             "hint, but steps may partly read it from L2"
                             if KV_BYTES_PER_TOKEN * args.context / world < 2 * L2_BYTES else ""))},
        "hbm_gbs_aggregate": total_bytes / (ms / K / 1e3) / 1e9,
        "per_rank": {"columns": ["step_us", "partial_us", "local_tokens"], "rows": per_rank_rows},
        "roofline": {"bound": "hbm", "kernel": "decode_step_kernel (+ combine of its splits)",
                     "achieved": local_bytes / (part_ms / 1e3) / 1e9, "peak": peak, "peak_source": peak_kind,
                     "unit": "GB/s", "frac": local_bytes / (part_ms / 1e3) / 1e9 / peak, "traffic": None,
                     "algorithmic_bytes": local_bytes, "avg_launch_ms": part_ms},
        "clocks": clocks.summary(),
        "gpu_launches": K * {"p2p": 2, "collective": 1 + (lc.splits > 16) + 2,
                             "direct": 1 + (lc.splits > 16)}[lc.exchange],
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph, graph_ev
    lc.close()
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def run_c1(args):
    """Config C1: one attention layer for one decode token of one sequence at
    --context cached tokens (512 by default here): x -> q/k/v projections
    (cuBLAS) -> fused step (norm + RoPE + append + attention) -> out_proj,
    the C1 layer of the golden fixtures.  value = steps per second (latency =
    ms_per_step); every step is the same token at the same position, so the
    cache does not grow.  Replicas across GPUs."""
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    attn = importlib.import_module(PKG + ".attention")
    pc = importlib.import_module(PKG + ".paged_cache")
    L = args.context if args.context != 131072 else 512
    cache = pc.PagedKVCache(pc.blocks_for(L + 1), L + 1, device=dev, shuffle_seed=args.seed * 1000 + 17)
    cache.add_sequence(L, capacity=L + 1)
    gen = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank + 29)
    cache.k.normal_(generator=gen)
    cache.v.normal_(generator=gen)
    w = synthetic_attention_weights(args.seed)
    wqkv = torch.cat([w["q_proj"], w["k_proj"], w["v_proj"]]).to(dev).contiguous()
    wo = w["out_proj"].to(dev).contiguous()
    runner = attn.PagedDecodeAttention(cache, w["q_gamma"], w["k_gamma"], 1, L + 2)
    x = torch.randn(1, 1024, generator=gen, device=dev).to(torch.bfloat16)
    qkv = torch.empty(1, 2048, dtype=torch.bfloat16, device=dev)
    y = torch.empty(1, 1024, dtype=torch.bfloat16, device=dev)
    past = torch.tensor([L], dtype=torch.int32, device=dev)
    seq, tables = past + 1, cache.block_tables()
    stream = torch.cuda.Stream(dev)

    def layer():
        torch.matmul(x, wqkv.t(), out=qkv)
        ctx = runner.step(0, qkv, past, seq, tables)
        torch.matmul(ctx.reshape(1, 1024), wo.t(), out=y)

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            layer()
    stream.synchronize()
    runner.check()
    K = args.steps
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(K):
            layer()
    graph.replay()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            t0.record()
            graph.replay()
            t1.record()
        torch.cuda.synchronize()
    runner.check()
    ms = t0.elapsed_time(t1)
    nbytes = KV_BYTES_PER_TOKEN * (L + 4) + 4 * pc.blocks_for(L + 1) + 2 * (2048 * 1024 + 1024 * 1024)
    peak, peak_kind = measured_hbm_peak()
    gbs = nbytes / (ms / K / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": K / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": K,
        "warmup": args.warmup, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "replicas",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"C1: one attention layer (q/k/v and out projections + fused decode step) for "
                               f"one token of one sequence at {L} cached tokens, CUDA graph of {K} steps",
                   "context": L, "global_batch": 1, "blocks_per_split": runner.blocks_per_split,
                   "parallelism": "replicas", "l2": "6 MB of weights and 1 MB of K/V stay in L2 across steps"},
        "hbm_gbs_per_gpu": gbs,
        "roofline": {"bound": "latency", "kernel": "qkv GEMM + decode_step_kernel + out GEMM",
                     "achieved": gbs, "peak": peak, "peak_source": peak_kind, "unit": "GB/s", "frac": gbs / peak,
                     "traffic": None, "algorithmic_bytes": nbytes},
        "clocks": clocks.summary(), "gpu_launches": K,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_c2(args):
    """Config C2: one sequence, the 6 attention layers of LFM2.5-230M, 64
    consecutive decode steps from --context cached tokens (each step appends
    one token per layer and attends over the grown cache).  One timed step =
    one token through the 6 layers; the 64-step run is captured once as a
    CUDA graph and replayed.  Replicas only across GPUs."""
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    L0 = args.context
    reps = max(1, args.steps // 64)
    clocks = ClockSampler(local)
    pt = c2_point(args, dev, L0, reps, sampler=clocks)
    peak, peak_kind = measured_hbm_peak()
    line = {
        "metric": METRIC, "value": pt["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1, "steps": reps * 64,
        "warmup": 3, "ms_per_step": pt["us_per_token"] / 1e3, "higher_is_better": True, "scaling": "replicas",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"C2: one sequence, 6 attention layers x 64 consecutive decode steps from "
                               f"{L0} cached tokens (CUDA graph of the 64 steps, replayed {reps}x)",
                   "context": L0, "global_batch": 1, "blocks_per_split": pt["blocks_per_split"],
                   "parallelism": "replicas", "l2": "K/V of 6 layers; the step re-reads its cache once"},
        "hbm_gbs_per_gpu": pt["gbs"], "hbm_pct_of_8tbs": 100 * pt["gbs"] / 8000,
        "roofline": {"bound": "hbm", "kernel": "decode_step_kernel x 6 layers", "achieved": pt["gbs"],
                     "peak": peak, "peak_source": peak_kind, "unit": "GB/s", "frac": pt["frac"], "traffic": None},
        "clocks": clocks.summary(), "gpu_launches": reps * 64 * 6 * (1 + (pt["splits"] > 16)),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


def c5_point(args, dev, rank: int = 0) -> dict:
    """One C5 run (see run_c5): ms for the whole job, its clocks and the
    generated ids' shape."""
    runner_mod = importlib.import_module(PKG + ".lfm2_runner")
    batch, prompt_len, new = 256, 32, 256
    sd = synthetic_lfm2_weights(args.seed, dev)
    runner = runner_mod.LFM2DecodeRunner(sd, max_batch=batch, max_context=prompt_len + new + 1, device=dev,
                                         fused_glue=not args.torch_glue,
                                         own_gemm=args.b2_gemm and not args.torch_glue)
    del sd
    g = torch.Generator().manual_seed(args.seed * 1000 + rank)
    prompts = torch.randint(0, 65536, (batch, prompt_len), generator=g)
    runner.generate(prompts[:, :4], 4)   # warm-up + graph capture
    torch.cuda.synchronize()
    runner.reset()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        t0.record()
        out = runner.generate(prompts, new)
        t1.record()
        torch.cuda.synchronize()
    runner.check()
    ms = t0.elapsed_time(t1)
    del runner
    torch.cuda.empty_cache()
    return {"ms": ms, "batch": batch, "prompt": prompt_len, "new": new, "shape": list(out.shape),
            "clocks": clocks.summary(), "tokens_per_s": batch * new / (ms / 1e3),
            "us_per_token_step": 1e3 * ms / (prompt_len + new - 1),
            "projections": "b2_gemm (tcgen05, SwiGLU fused into w1/w3)" if args.b2_gemm and not args.torch_glue
            else "cuBLAS (torch.matmul)",
            "layer_glue": "torch ops" if args.torch_glue else "libb2attn kernels"}


def run_c5(args):
    """Config C5: end-to-end greedy decode of an LFM2.5-230M-shaped random-init
    model (14 layers: 8 short-conv + 6 GQA attention, SwiGLU 2560, tied 65536
    head): 256 prompts x 32 random ids, 256 new tokens each, paged KV, one
    CUDA graph per token.  value = new tokens per second over the whole job
    (prefill included); replicas across GPUs (each rank its own batch)."""
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pt = c5_point(args, dev, rank)
    batch, prompt_len, new, ms = pt["batch"], pt["prompt"], pt["new"], pt["ms"]
    line = {
        "metric": METRIC, "value": batch * new / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
        "steps": prompt_len + new - 1, "warmup": 1, "ms_per_step": ms / (prompt_len + new - 1),
        "higher_is_better": True, "scaling": "replicas", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "C5 end-to-end greedy decode, LFM2.5-230M-shaped random-init model, "
                               "256 prompts x 32 ids, 256 new tokens, paged KV, CUDA graph per token",
                   "layer_glue": "torch ops" if args.torch_glue else "libb2attn kernels",
                   "projections": "b2_gemm (tcgen05, SwiGLU fused into w1/w3)" if args.b2_gemm and not args.torch_glue
                   else "cuBLAS (torch.matmul)",
                   "global_batch": batch * world, "prompt": prompt_len, "new_tokens": new,
                   "parallelism": f"replicas x{world}"},
        "generated_shape": pt["shape"], "clocks": pt["clocks"],
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


def prefill_point(args, dev, T, K, W, rank=0, path="prefill"):
    """K steps of the batched prompt (a CUDA graph; the K/V pool, 0.5 GB,
    exceeds L2): the C3 batch of 64 sequences with cached prefixes
    L ~ U[128, 8192], each receiving T new tokens through one attention layer
    (append of the chunk + tcgen05 attention; path "step": the fused decode
    step for T <= 4 new tokens, b2_decode_step_tokens).  Returns the timing,
    the HBM figures and the clocks."""
    attn = importlib.import_module(PKG + ".attention")
    pc = importlib.import_module(PKG + ".paged_cache")
    rope = importlib.import_module(PKG + ".rope")
    lengths = seq_lengths(args, 0)
    caps = [n + T for n in lengths]
    cache = pc.PagedKVCache(sum(pc.blocks_for(c) for c in caps), max(caps), device=dev,
                            shuffle_seed=args.seed * 1000 + 17)
    for n, c in zip(lengths, caps):
        cache.add_sequence(n, capacity=c)
    gen = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank + 29)
    cache.k.normal_(generator=gen)
    cache.v.normal_(generator=gen)
    gg = torch.Generator().manual_seed(args.seed + 31)
    gq = (1.0 + 0.1 * torch.randn(D, generator=gg)).to(torch.bfloat16).to(dev)
    gk = (1.0 + 0.1 * torch.randn(D, generator=gg)).to(torch.bfloat16).to(dev)
    cos, sin = rope.rope_table(max(caps) + 1, device=dev)
    b = len(lengths)
    qkv = (torch.randn(b, T, 2048, generator=gen, device=dev) * 0.6).to(torch.bfloat16)
    past = torch.tensor(lengths, dtype=torch.int32, device=dev)
    tables = cache.block_tables()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    q_out = torch.empty(b, T, HQ, D, dtype=torch.bfloat16, device=dev)
    out = torch.empty(b, T, HQ, D, dtype=torch.bfloat16, device=dev)
    kp, vp = cache.pool(0)
    stream = torch.cuda.Stream(dev)
    if path == "step":
        bps = attn.step_tokens_blocks_per_split(b, tables.shape[1])
        counters = torch.zeros(2 + 8 * b, dtype=torch.int32, device=dev)
        splits = attn.num_splits_for(tables.shape[1], bps)
        part_ml = torch.empty(b, T, splits, HQ, 2, dtype=torch.float32, device=dev)
        part_o = torch.empty(b, T, splits, HQ, D, dtype=torch.float32, device=dev)

        def step():
            attn.decode_step_tokens(qkv, past, k_pool=kp, v_pool=vp, block_tables=tables, out=out,
                                    counters=counters, dev_err=err, blocks_per_split=bps, part_ml=part_ml,
                                    part_o=part_o, gamma_q=gq, gamma_k=gk, cos=cos, sin=sin, q_out=q_out)
    else:
        bps = attn.prefill_blocks_per_split(b, T, tables.shape[1]) if args.prefill_bps < 0 else args.prefill_bps

        def step():
            attn.prefill(qkv, past, k_pool=kp, v_pool=vp, block_tables=tables, gamma_q=gq, gamma_k=gk, cos=cos,
                         sin=sin, dev_err=err, out=out, q_out=q_out,
                         blocks_per_split=None if args.prefill_bps < 0 else args.prefill_bps, kernel="tcgen05")

    with torch.cuda.stream(stream):
        for _ in range(max(W, 1)):
            step()
    torch.cuda.synchronize()
    assert err.item() == 0, "device error in prefill"
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(K):
            step()
    graph.replay()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index or 0) as clocks:
        with torch.cuda.stream(stream):
            t0.record()
            graph.replay()
            t1.record()
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / K
    assert err.item() == 0, "device error in prefill"
    nbytes = sum(KV_BYTES_PER_TOKEN * (n + T) + T * (2048 * 2 + HQ * D * 2 * 2) for n in lengths)
    # useful flops: each chunk token's 16 heads over the keys it sees (causal)
    flops = sum(4 * HQ * D * sum(n + t + 1 for t in range(T)) for n in lengths)
    peak, peak_kind = measured_hbm_peak()
    gbs = nbytes / (ms / 1e3) / 1e9
    del graph
    return {"batch": b, "chunk": T, "ms": ms, "tokens_per_s": b * T / (ms / 1e3), "gbs": gbs,
            "frac": gbs / peak, "peak": peak, "peak_kind": peak_kind, "bytes": nbytes,
            "tflops": flops / (ms / 1e3) / 1e12, "blocks_per_split": bps, "clocks": clocks.summary()}


def prefill_points(args, dev) -> dict:
    """The batched-prompt kernel beside the decode line (the reference's x8p
    4-token prompt batches, and 64 / 128-token chunks): 64 sequences x T."""
    rows = []
    for T, path in ((4, "prefill"), (64, "prefill"), (128, "prefill"), (4, "step")):
        pt = prefill_point(args, dev, T, 20, 3, path=path)
        rows.append({"chunk": T, "kernel": "decode_step_kernel (b2_decode_step_tokens)" if path == "step"
                     else "prefill_attn_kernel (tcgen05)", "us_per_step": round(pt["ms"] * 1e3, 2),
                     "tokens_per_s": round(pt["tokens_per_s"], 1), "gbs": round(pt["gbs"], 1),
                     "frac": round(pt["frac"], 4), "blocks_per_split": pt["blocks_per_split"]})
        torch.cuda.empty_cache()
    return {"note": "batched prompt: the C3 batch (64 sequences, cached L ~ U[128, 8192]) each receiving "
                    "`chunk` new tokens through one attention layer (chunk append + tcgen05 attention, "
                    "causal within the chunk); frac of the measured HBM copy peak over K/V read once",
            "points": rows}


def run_prefill(args):
    """Batched-prompt attention (the x8p engine's batched prompt tile, grown to
    64-token chunks): the C3 batch of 64 sequences with cached prefixes
    L ~ U[128, 8192], each receiving --chunk new tokens through one attention
    layer (append of the chunk + tcgen05 attention; --prefill-kernel step: the
    fused decode step for chunks of up to 4 tokens).  tokens/s counts chunk
    tokens.  Replicas across GPUs."""
    T, K = args.chunk, args.steps
    step = args.prefill_kernel == "step"
    if step and not 1 <= T <= 4:
        raise SystemExit("--prefill-kernel step takes chunks of 1-4 tokens")
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pt = prefill_point(args, dev, T, K, args.warmup, rank, path="step" if step else "prefill")
    ms, gbs, peak = pt["ms"], pt["gbs"], pt["peak"]
    kernel = "decode_step_kernel" if step else "append_rope_kernel + prefill_attn_kernel"
    line = {
        "metric": METRIC, "value": pt["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1, "steps": K,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "replicas",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"batched prompt: 64 sequences with cached L ~ U[128, 8192] each receiving "
                               f"{T} new tokens through one attention layer ("
                               + ("fused decode step: norm + RoPE + append + attention + merge in one launch"
                                  if step else "chunk append + tcgen05 attention")
                               + ", causal within the chunk)", "chunk": T, "kernel": args.prefill_kernel,
                   "prefill_blocks_per_split": pt["blocks_per_split"],
                   "global_batch": pt["batch"], "parallelism": "replicas"},
        "hbm_gbs_per_gpu": gbs, "tflops": pt["tflops"],
        "roofline": {"bound": "hbm", "kernel": kernel, "achieved": gbs,
                     "peak": peak, "peak_source": pt["peak_kind"], "unit": "GB/s", "frac": gbs / peak,
                     "traffic": None, "algorithmic_bytes": pt["bytes"]},
        "clocks": pt["clocks"], "gpu_launches": (1 if step else 2) * K,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world, _, _ = dist_env()
    if world != args.gpus and not (world == 1 and args.gpus == 1):
        if world == 1 and args.gpus > 1:
            raise SystemExit("--gpus N > 1 must be launched with torchrun (one process per GPU)")
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "c4":
        run_c4(args)
    elif args.config == "c1":
        run_c1(args)
    elif args.config == "c2":
        run_c2(args)
    elif args.config == "c5":
        run_c5(args)
    elif args.config == "prefill":
        run_prefill(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
