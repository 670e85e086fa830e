#!/usr/bin/env python
"""Decode throughput of the tensor-parallel decoder-layer forward on B200.

Workload (default): the Llama-3-8B shape (hidden 4096, 32 layers, 32 q / 8 kv heads,
intermediate 14336, vocab 128256), bf16, decoding a batch of 128 sequences at
context 2048 in the paged KV cache (block_size 16, block tables a seeded random
permutation of the pool), tensor parallel over N GPUs (one process per GPU; the
row-parallel all-reduce runs over NVLink peer memory).  Weights are N(0, 0.02)
and the KV cache is random (synthetic data; there is no checkpoint or dataset).

  python bench.py --gpus N --steps K --warmup W           # this framework
  python bench.py --impl reference --steps K --warmup W   # the reference's CPU path (restated)
  python bench.py --workload prefill                      # batched varlen prefill (below)
  python bench.py --workload mixed                        # 16 x 1024 prefills + 240 decodes in one step
  python bench.py --workload tinyllama                    # TinyLlama, 64 requests x 128 new tokens
  torchrun --nproc-per-node N bench.py --workload allreduce   # row-parallel all-reduce (below)

Before timing, the decode workload checks an 8B-shape layer at this TP degree against
the oracle's fixture and, at TP <= 2, the Tiny LLaMA tokens against the reference's own
(the ``parity`` object; a failure exits non-zero).  At TP > 1 the line also carries the
row-parallel sweep (``fused_allreduce_sweep``: T in 1..4096 against NCCL).

One JSON line on rank 0:
  value        decode tokens/s with inputs resident in HBM (CUDA events, max over ranks)
  e2e          the same through WorkerExecutionEngine.execute_step with host-side
               StepRequests: pinned H2D of the step's inputs and D2H of the sampled
               tokens and top logits inside the timed region
  roofline     the dominant kernel's achieved HBM GB/s vs the measured copy peak
  cpu_baseline the reference's CPU path restated on torch CPU (oracle/grpc_tp.py) on
               this host's cores: one decoder layer of the full batch plus 1/8 of
               the lm_head, extrapolated to a full step (rank 0 at N=1); the
               reference arm runs it at TP = N over the reference's gRPC all-reduce

``--workload prefill`` measures the other half of a serving step instead: the
Mistral-7B shape (vocab 32000), 16 prompts of 1024 tokens prefilled in ONE batched
forward (the reference runs one forward per prompt), metric prefill tokens/s; the
roofline is the dominant kernel's TFLOP/s against the bf16 tensor peak.

``--workload allreduce`` (N >= 2 ranks) is the row-parallel microbenchmark: bf16
X [T, 14336/N] x W [14336/N, 4096], then all-reduce(SUM) + float32 residual + RMSNorm,
for T in 1, 8, 64, 512, 4096, as ONE fused pair of launches (the GEMM epilogue pushes
partial rows to their owners over NVLink; the owners reduce, normalise and all-gather).
Metric: bus GB/s = 2 (N - 1) / N * T * 4096 * 2 B / time at T = 4096, beside an NCCL
all-reduce of the same payload and the GEMM alone.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

HBM_FALLBACK_GBS = 6650.0
BF16_FALLBACK_TFLOPS = 1590.0

# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) over the
# algorithmic bytes of the same launch, from one ncu capture of the attention kernel at
# batch 128, context 2048: 1.0887 GB measured for 1.0884 GB algorithmic.  Traffic grows with the KV bytes read,
# so other batch sizes, contexts and TP degrees scale it by their algorithmic bytes.
MEASURED_TRAFFIC_RATIO = {"paged_attention": 1.0887e9 / 1088421888}


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=32, help="decoder layers (32 = the full model)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the TP parity leg (it runs before timing)")
    ap.add_argument("--no-sweep", action="store_true", help="skip the row-parallel sweep at TP > 1")
    ap.add_argument("--workload", choices=["decode", "prefill", "allreduce", "mixed", "tinyllama"], default="decode")
    ap.add_argument("--prompts", type=int, default=16, help="prefill workload: prompts per step")
    ap.add_argument("--prompt-len", type=int, default=1024, help="prefill workload: tokens per prompt")
    return ap.parse_args(argv)


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


def measured_tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured"
    except Exception:
        return BF16_FALLBACK_TFLOPS, "fallback"


def init_synthetic(model, pool, seed: int, rank: int, dev):
    """N(0, 0.02) weights (norms 1), identical replicated tensors on every rank, and a random KV cache."""
    import torch
    g_rep = torch.Generator(device=dev)
    g_rep.manual_seed(seed)
    g_shard = torch.Generator(device=dev)
    g_shard.manual_seed(seed + 1 + rank)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "layernorm" in name or name == "norm.weight":
                p.fill_(1.0)
                continue
            replicated = name.startswith("embed_tokens") or name.startswith("lm_head")
            p.normal_(0.0, 0.02, generator=g_rep if replicated else g_shard)
        pool.k_cache.normal_(0.0, 1.0, generator=g_shard)
        pool.v_cache.normal_(0.0, 1.0, generator=g_shard)


def model_config(layers: int):
    from pythonintern_b200 import workloads
    return workloads.llama3_8b_config(num_layers=layers, max_seq_len=4096)


def workload_name(args, n):
    full = " (full 32 layers)" if args.layers == 32 else f" ({args.layers} layers)"
    return f"llama3-8b-shape decode, batch {args.batch}, context {args.ctx}, TP={n}{full}"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clocks and throttle reasons sampled every 10 ms (NVML, in a thread) during the timed region.

    Falls back to ``nvidia-smi -lms 50`` when NVML cannot be loaded.  A short timed region
    (a few tens of milliseconds at TP=8) still gets several samples this way.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits (nvml.h): sw power cap 0x4, hw slowdown 0x8,
    # sw thermal 0x20, hw thermal 0x40.
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu_index: int, period_s: float = 0.01):
        self.gpu = gpu_index
        self.period = period_s
        self.proc = None
        self.path = None
        self.thread = None
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self.stop_flag = None

    def start(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
            self.stop_flag = threading.Event()

            def loop():
                while not self.stop_flag.is_set():
                    try:
                        self.samples.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                        bits = int(reasons_fn(h))
                        for nm, b in self.BITS.items():
                            if bits & b:
                                self.reasons.add(nm)
                    except Exception:
                        pass
                    self.stop_flag.wait(self.period)
            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        fd, self.path = tempfile.mkstemp(prefix="b2clk", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=2)
            sm = self.samples
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                    "reasons": sorted(self.reasons), "samples": len(sm), "source": "NVML, 10 ms period"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for nm, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(nm)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi, 50 ms period"}


# ----------------------------------------------------------------------------- CPU leg
def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_decode(cfg, world: int, batch: int, ctx: int, steps: int, warmup: int, seed: int, cores: int):
    """The reference's CPU decode, restated on torch CPU (oracle/grpc_tp.py), timed on this host.

    ``world`` rank processes (``cores // world`` threads each) each run their shard of ONE
    decoder layer of ``cfg``'s shape for ``batch`` sequences at context ``ctx`` (paged pool,
    permuted block tables, zero padding, repeat_kv, float32), joined by the reference's
    gRPC all-reduce after out_proj and down_proj, plus 1/8 of the replicated lm_head.
    Returns the oracle timing dict: per-step seconds extrapolated to all layers and the
    whole lm_head (max over ranks), the sampled wall times and the thread counts.
    """
    from oracle import grpc_tp
    return grpc_tp.time_tp_decode(world, cfg.hidden_dim, cfg.num_heads, cfg.num_kv_heads, cfg.intermediate_dim,
                                  cfg.vocab_size, cfg.num_layers, batch, ctx, steps, warmup, seed, cores)


def cpu_sample_text(cfg, world, batch, ctx, r):
    ex = (f"; the {world} rank processes exchange partial sums over the reference's gRPC all-reduce "
          f"(protobuf AllReducePayload on localhost)") if world > 1 else ""
    return (f"torch-CPU restatement of the reference's float32 decode path: {batch} sequences at context {ctx}, "
            f"1 of {cfg.num_layers} decoder layers + 1/{round(cfg.vocab_size / r['vocab_slice'])} of the lm_head "
            f"timed per step and extrapolated to the full step; TP={world}, {r['threads_per_rank']} threads per "
            f"rank{ex}")


def cpu_baseline_entry(args, cfg):
    """Bounded sample for the GPU arm's line (rank 0 at N=1): one warm-up and one timed step."""
    cores = cpu_cores()
    r = cpu_decode(cfg, 1, args.batch, args.ctx, 1, 1, args.seed, cores)
    t = statistics.median(r["step_s"])
    return {"value": args.batch / t, "unit": "tokens/s", "cores": sum(r["threads_used"]), "kind": "port",
            "sample": cpu_sample_text(cfg, 1, args.batch, args.ctx, r), "batch": args.batch, "layers_sampled": 1,
            "sample_s": r["sample_wall_s"][0]}


def run_reference_prefill(args):
    """Reference arm of the prefill workload: the oracle's one-prompt-per-forward prefill."""
    from pythonintern_b200 import workloads
    cfg = workloads.mistral_7b_config(num_layers=32)
    n, P = args.prompts, args.prompt_len
    for _ in range(max(0, args.warmup)):
        cpu_prefill_sample(cfg, P, args.seed)
    times = [cpu_prefill_sample(cfg, P, args.seed) * cfg.num_layers * n for _ in range(max(1, args.steps))]
    t = statistics.median(times)
    value = n * P / t
    sample = (f"per step: one prompt of {P} tokens through 1 of {cfg.num_layers} decoder layers, extrapolated to "
              f"{n} prompts x {cfg.num_layers} layers; median of {len(times)} steps")
    line = {
        "impl": "reference", "metric": "prefill tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1000.0,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"mistral-7b-shape batched prefill, {n} prompts x {P} tokens, TP=1 (CPU)",
                   "model": "mistral-7b-shape", "global_batch": n, "seq_len": P, "parallelism": "tp1 (CPU)"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cpu_cores(), "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference(args):
    """Reference arm: the reference's CPU path (restated, oracle/grpc_tp.py) on this host's cores.

    Under torchrun only rank 0 works; it starts ``world`` CPU rank processes itself (the
    reference runs one worker process per shard) and splits the host's cores among them.
    """
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return 0
    if args.workload == "prefill":
        return run_reference_prefill(args)
    if args.workload == "allreduce":
        return run_reference_allreduce(args, world)
    cfg = model_config(32)
    cores = cpu_cores()
    r = cpu_decode(cfg, world, args.batch, args.ctx, max(1, args.steps), max(0, args.warmup), args.seed, cores)
    t = statistics.median(r["step_s"])
    value = args.batch / t
    line = {
        "impl": "reference", "metric": "decode tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1000.0,
        "sample_ms_per_step": statistics.median(r["sample_wall_s"]) * 1000.0,
        "ms_per_step_note": ("ms_per_step is the full 32-layer step extrapolated from the timed sample "
                             "(1 decoder layer + 1/8 of the lm_head per step); sample_ms_per_step is the wall "
                             "time each timed step actually took"),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: N(0,0.02) weights, random KV cache, random block-table permutation",
        "config": decode_config(args, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": sum(r["threads_used"]), "kind": "port",
                         "sample": cpu_sample_text(cfg, world, args.batch, args.ctx, r) +
                         f"; median of {len(r['step_s'])} steps",
                         "batch": args.batch, "layers_sampled": 1, "threads_per_rank": r["threads_per_rank"],
                         "ranks": world, "host_cores": cores},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


ROWPAR_TOKENS = (1, 8, 64, 512, 4096)


def run_reference_allreduce(args, world):
    """Reference arm of the row-parallel microbenchmark: float32 partial GEMM + gRPC all-reduce +
    residual + RMSNorm across ``world`` CPU rank processes (the reference has no bf16 path)."""
    if world < 2:
        print(json.dumps({"impl": "reference", "metric": "row-parallel all-reduce bus GB/s",
                          "unavailable": "needs >= 2 ranks (torchrun --nproc-per-node N)"}), flush=True)
        return 0
    from oracle import grpc_tp
    H, I = 4096, 14336
    cores = cpu_cores()
    r = grpc_tp.time_row_parallel(world, ROWPAR_TOKENS, H, I, args.seed, cores)
    rows = []
    for T, t in zip(ROWPAR_TOKENS, r["s"]):
        nbytes = T * H * 4
        rows.append({"tokens": T, "payload_bytes": nbytes, "us": t * 1e6,
                     "bus_gbs": 2 * (world - 1) / world * nbytes / t / 1e9})
    top = rows[-1]
    line = {
        "impl": "reference", "metric": "row-parallel all-reduce bus GB/s", "value": top["bus_gbs"], "unit": "GB/s",
        "n_gpus": world, "steps": None, "warmup": 1, "ms_per_step": top["us"] / 1000.0,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded activations, N(0,0.02) weights",
        "config": rowpar_config(world),
        "cpu_baseline": {"value": top["bus_gbs"], "unit": "GB/s", "cores": sum(r["threads_used"]), "kind": "port",
                         "sample": (f"torch-CPU restatement of RowParallelLinear.forward + the reference's gRPC "
                                    f"all-reduce across {world} rank processes ({r['threads_per_rank']} threads each) "
                                    f"+ residual + RMSNorm, float32 payload (the reference has no bf16 path); best "
                                    f"of 3 calls (1 at 4096 tokens) after one warm-up")},
        "e2e": {"value": top["bus_gbs"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "sizes": rows,
    }
    print(json.dumps(line), flush=True)
    return 0


def decode_config(args, world):
    return {"workload": workload_name(args, world), "model": "llama3-8b-shape", "global_batch": args.batch,
            "seq_len": args.ctx, "parallelism": f"tp{world}",
            "l2": "inputs larger than L2 (weights + KV read per step >> 126 MB)"}


def rowpar_config(world):
    return {"workload": (f"row-parallel GEMM [T, 14336/{world}] x [14336/{world}, 4096] + all-reduce + residual "
                         f"+ RMSNorm, TP={world}; value at T=4096"),
            "parallelism": f"tp{world}", "tokens": list(ROWPAR_TOKENS)}


# ----------------------------------------------------------------------------- parity leg
PARITY_FIXTURE = os.path.join(ROOT, "tests", "golden", "llama3_8b_layer_parity.npz")
PARITY_TOL = 2e-2  # bf16: relative Frobenius error of the residual stream after the layer


def tp_parity(comm, rank: int, world: int, dev) -> dict:
    """Checks the CUDA path at TP=world against committed fixtures before anything is timed.

    * One Llama-3-8B-shape decoder layer (vocabulary 4096, seeded N(0, 0.02) weights
      sharded by WeightSharder): two prompts of 40 and 13 tokens prefilled in one varlen
      call, then two batched decode steps fed the fixture's tokens.  The residual stream
      after the layer, gathered over the ranks' row slices, must be within relative 2e-2
      of the oracle's (tests/golden/llama3_8b_layer_parity.npz, made by
      tests/golden/make_tp_parity.py); the greedy tokens (vocab-parallel exchange at
      TP>1) must equal the oracle's wherever its top-2 margin exceeds the measured logit
      error, and be identical on every rank.
    * At TP=1 and TP=2, the float32 Tiny LLaMA workload (8 requests, 32 greedy steps
      through execute_step) must give exactly the tokens the reference itself produced
      (tests/golden/tiny_e2e_tp{1,2}.npz).
    Every rank takes the same collective steps; the result is the same dict on all ranks.
    """
    import torch
    import torch.distributed as dist

    from pythonintern_b200 import _lib, workloads
    from pythonintern_b200.model.kv_cache import PhysicalKVCachePool
    from pythonintern_b200.model.llama import DistributedLLaMAModel
    from pythonintern_b200.model.metadata import build_metadata, build_prefill_metadata
    from pythonintern_b200.tensor_parallel.sharding import WeightSharder

    fx = np.load(PARITY_FIXTURE)
    cfg = workloads.llama3_8b_config(num_layers=1, max_seq_len=512)
    cfg.vocab_size = 4096
    sd = WeightSharder(cfg, world).shard_full_model_state_dict(workloads.synthetic_state_dict(cfg, seed=21), rank)
    model = DistributedLLaMAModel(cfg, rank, world, comm, device=dev)
    model.load_state_dict(sd)
    del sd
    pool = PhysicalKVCachePool(16, 16, max(1, cfg.num_kv_heads // world), cfg.head_dim, 1, dev, "bfloat16")
    prompts = [fx["prompt0"], fx["prompt1"]]
    lens = [int(p.size) for p in prompts]
    tables = [[3, 9, 1, 12], [5, 0]]
    err2 = torch.zeros((), dtype=torch.float64, device=dev)
    ref2 = torch.zeros((), dtype=torch.float64, device=dev)
    logit_err = 0.0
    toks_gpu, toks_fwd = [], []

    def accumulate(tr, ref):
        nonlocal err2, ref2
        if world > 1:
            r0, rows = tr
        else:
            r0, rows = 0, tr
        n = rows.shape[0]
        if n == 0:  # at TP > 1 a rank can own none of a short batch's rows
            return
        want = torch.from_numpy(ref[r0:r0 + n].astype(np.float32)).to(dev, torch.float64)
        got = rows.reshape(n, want.shape[1]).to(torch.float64)
        err2 += (got - want).pow(2).sum()
        ref2 += want.pow(2).sum()

    with torch.no_grad():
        ids = torch.from_numpy(np.concatenate(prompts)[None]).to(dev)
        md = build_prefill_metadata(lens, tables, dev)
        tr = []
        logits = model(ids, None, pool, tables, True, 0, metadata=md, trace=tr)
        accumulate(tr[0], fx["hidden_prefill"])
        logit_err = max(logit_err, float((logits.cpu() - torch.from_numpy(fx["logits"][0])).abs().max()))
        toks_fwd.append(logits.argmax(-1).cpu())
        tok, _ = model.greedy(ids, None, pool, tables, True, 0, metadata=md)
        toks_gpu.append(tok.view(-1).cpu())
        for s in range(2):
            feed = torch.from_numpy(fx["tokens"][s]).view(2, 1).to(dev)
            pos = torch.tensor([[lens[0] + s], [lens[1] + s]])
            md = build_metadata(pos, tables, False, dev)
            tr = []
            logits = model(feed, pos, pool, tables, False, s + 1, metadata=md, trace=tr)
            accumulate(tr[0], fx["hidden_decode"][s])
            logit_err = max(logit_err, float((logits.cpu() - torch.from_numpy(fx["logits"][s + 1])).abs().max()))
            toks_fwd.append(logits.argmax(-1).cpu())
            tok, _ = model.greedy(feed, pos, pool, tables, False, s + 1, metadata=md)
            toks_gpu.append(tok.view(-1).cpu())
        torch.cuda.synchronize(dev)
        _lib.check_device_status(dev, "parity layer")
    gpu_tok = torch.stack(toks_gpu).to(dev)
    stats = torch.stack([err2, ref2])
    lerr = torch.tensor([logit_err], dtype=torch.float64, device=dev)
    tmax, tmin = gpu_tok.clone(), gpu_tok.clone()
    if world > 1:
        dist.all_reduce(stats)
        dist.all_reduce(lerr, op=dist.ReduceOp.MAX)
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(tmin, op=dist.ReduceOp.MIN)
    rel = float((stats[0] / stats[1]).sqrt())
    logit_err = float(lerr.item())
    bound = max(0.05, 3.0 * logit_err)
    sel = fx["margins"] > bound
    want_tok = fx["tokens"]
    got = gpu_tok.cpu().numpy()
    fwd = torch.stack(toks_fwd).numpy()
    tokens_match = bool(np.array_equal(got[sel], want_tok[sel]) and np.array_equal(fwd[sel], want_tok[sel]))
    ranks_agree = bool(torch.equal(tmax, tmin))
    del model, pool
    out = {"tp": world, "layer": ("llama3-8b shape, 1 layer, vocab 4096; prefill of 40 + 13 tokens, 2 decode steps; "
                                  "oracle fixture tests/golden/llama3_8b_layer_parity.npz"),
           "layer_rel_err": rel, "tol": PARITY_TOL, "logits_max_abs_err": logit_err,
           "tokens_checked": int(sel.sum()), "tokens_total": int(sel.size), "token_margin_bound": bound,
           "tokens_match": tokens_match, "ranks_agree": ranks_agree, "tiny_tokens_match": None}
    if world <= 2:
        out["tiny_tokens_match"] = tiny_tokens_check(comm, rank, world, dev)
        out["tiny"] = f"Tiny LLaMA float32, 8 requests x 32 greedy steps vs the reference's own TP={world} tokens"
    torch.cuda.empty_cache()
    out["pass"] = bool(rel < PARITY_TOL and tokens_match and ranks_agree and out["tiny_tokens_match"] is not False)
    return out


def tiny_tokens_check(comm, rank: int, world: int, dev) -> bool:
    """The Tiny LLaMA greedy workload through execute_step; True if the tokens equal the golden."""
    import torch
    import torch.distributed as dist

    from pythonintern_b200 import workloads
    from pythonintern_b200.config import KVCacheConfig, ShardConfig
    from pythonintern_b200.tensor_parallel.sharding import WeightSharder
    from pythonintern_b200.worker.execution_engine import WorkerExecutionEngine
    from pythonintern_b200.worker.messages import SequenceSlot, StepRequest

    gold = np.load(os.path.join(ROOT, "tests", "golden", f"tiny_e2e_tp{world}.npz"))
    cfg = workloads.tiny_config()
    eng = WorkerExecutionEngine(cfg, ShardConfig(rank, world), KVCacheConfig(16, 64, str(dev)), comm, dev)
    full = workloads.reference_init_state_dict(cfg, 0)
    eng.model.load_state_dict(WeightSharder(cfg, world).shard_full_model_state_dict(full, rank))
    prompts = workloads.tiny_prompts()
    ids = [f"req_{i}" for i in range(len(prompts))]
    for sid, p in zip(ids, prompts):
        eng.kv_manager.allocate_blocks_for_sequence(sid, len(p))
    lens = {sid: len(p) for sid, p in zip(ids, prompts)}
    cur, toks_all = {}, []
    for step in range(gold["tokens"].shape[0]):
        if step == 0:
            slots = [SequenceSlot(sid, True, p, 0, len(p), list(eng.kv_manager.block_tables[sid].physical_block_ids))
                     for sid, p in zip(ids, prompts)]
        else:
            slots = []
            for sid in ids:
                eng.kv_manager.append_token(sid)
                lens[sid] += 1
                slots.append(SequenceSlot(sid, False, [], cur[sid], lens[sid],
                                          list(eng.kv_manager.block_tables[sid].physical_block_ids)))
        resp = eng.execute_step(StepRequest(step, slots))
        toks = [t.token_id for t in resp.sampled_tokens]
        cur = dict(zip(ids, toks))
        toks_all.append(toks)
    ok = torch.tensor([1 if np.array_equal(np.asarray(toks_all), gold["tokens"]) else 0], device=dev)
    del eng
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    return bool(ok.item())


# ----------------------------------------------------------------------------- row-parallel sweep
def allreduce_sweep(comm, rank: int, world: int, dev, seed: int, tokens=None) -> dict:
    """Row-parallel GEMM [T, 14336/N] x [14336/N, 4096] + all-reduce + residual + RMSNorm per T,
    as the fused pair of launches, beside the GEMM alone and an NCCL all-reduce of the same
    payload (all device-timed in CUDA graphs or back-to-back launches, max over ranks), plus
    NCCL's all-reduce bus bandwidth at 256 MB as the measured NVLink reference."""
    import torch
    import torch.distributed as dist

    from pythonintern_b200 import _lib, kernels
    H, I = 4096, 14336
    K = I // world
    g = torch.Generator(device=dev)
    g.manual_seed(seed + 1 + rank)
    w = (torch.randn(H, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)  # packed [out, in] rows
    nw = torch.ones(H, device=dev)
    stream = torch.cuda.current_stream(dev)

    def max_over_ranks(x: float) -> float:
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def time_graph(fn, n, reps=5):
        for _ in range(2):
            fn()
        torch.cuda.synchronize(dev)
        dist.barrier()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for _ in range(n):
                fn()
        dist.barrier()
        gr.replay()
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            gr.replay()
        e1.record(stream)
        e1.synchronize()
        del gr
        return max_over_ranks(e0.elapsed_time(e1) / (reps * n) / 1000.0)

    def time_nccl(payload, n):
        for _ in range(3):
            dist.all_reduce(payload)
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            dist.all_reduce(payload)
        e1.record(stream)
        e1.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / n / 1000.0)

    rows = []
    for T in (tokens or ROWPAR_TOKENS):
        x = torch.randn(T, K, device=dev, generator=g).to(torch.bfloat16)
        r0, r1, R = comm.row_slice(T)
        h = torch.zeros(R, H, device=dev)
        y = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
        n = 20 if T <= 512 else 6  # an even count keeps the exchange slots in step

        def fused():
            comm.row_parallel_linear(x, w)
            comm.allreduce_rmsnorm_sharded(T, H, torch.bfloat16, h, nw, 1e-5, out=y)
        t_fused = time_graph(fused, n)
        t_gemm = time_graph(lambda: kernels.linear(x, w), n)
        t_nccl = time_nccl(torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16), n)
        nbytes = T * H * 2
        bus = 2 * (world - 1) / world * nbytes
        rows.append({"tokens": T, "payload_bytes": nbytes, "fused_us": t_fused * 1e6, "gemm_alone_us": t_gemm * 1e6,
                     "fused_bus_gbs": bus / t_fused / 1e9, "nccl_allreduce_us": t_nccl * 1e6,
                     "nccl_bus_gbs": bus / t_nccl / 1e9, "gemm_plus_nccl_us": (t_gemm + t_nccl) * 1e6,
                     "exchange_us": (t_fused - t_gemm) * 1e6})
        del x, h, y
    big = torch.empty(128 << 20, dtype=torch.bfloat16, device=dev)  # 256 MB
    t_big = time_nccl(big, 5)
    del big
    torch.cuda.empty_cache()
    _lib.check_device_status(dev, "row-parallel sweep")
    peak = 2 * (world - 1) / world * (256 << 20) / t_big / 1e9
    return {"sizes": rows, "nvlink_peak_gbs": peak,
            "nvlink_peak_source": f"NCCL all-reduce bus bandwidth at 256 MB, TP={world}, measured in this run",
            "note": ("fused_us includes the GEMM (its epilogue pushes the partial rows); bus GB/s counts the "
                     "all-reduce payload only; gemm_plus_nccl_us is the unfused alternative (GEMM, then an NCCL "
                     "all-reduce, without the residual and RMSNorm); exchange_us = fused_us - gemm_alone_us")}


# ----------------------------------------------------------------------------- GPU leg
def run_ours(args):
    import torch
    import torch.distributed as dist

    from pythonintern_b200 import _lib, kernels
    from pythonintern_b200.config import KVCacheConfig, ShardConfig
    from pythonintern_b200.model.metadata import build_metadata
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    from pythonintern_b200.worker.execution_engine import WorkerExecutionEngine
    from pythonintern_b200.worker.graphs import DecodeGraph, table_bucket
    from pythonintern_b200.worker.messages import SequenceSlot, StepRequest

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and rank == 0:
        print(f"note: WORLD_SIZE={world} but --gpus={args.gpus}; using WORLD_SIZE", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=dev)
    cfg = model_config(args.layers)
    B, ctx, W, K = args.batch, args.ctx, args.warmup, args.steps
    comm = None
    if world > 1:
        # 64 MB holds the row-parallel sweep's largest partial (4096 tokens x 4096 bf16)
        comm = DistributedCommunicator(rank, world, device=dev, max_bytes=max(64 << 20, B * cfg.hidden_dim * 2 * 2))
        comm.connect()
    parity = None if args.no_parity else tp_parity(comm, rank, world, dev)
    bps = math.ceil((ctx + W + K + 2 * (W + K) + 8) / 16)
    num_blocks = B * bps
    engine = WorkerExecutionEngine(cfg, ShardConfig(rank=rank, world_size=world),
                                   KVCacheConfig(block_size=16, num_blocks=num_blocks, device=str(dev)), comm, dev)
    model, pool = engine.model, engine.kv_manager.pool

    # Synthetic weights: replicated tensors identical on every rank, shards per rank.
    init_synthetic(model, pool, args.seed, rank, dev)
    perm = np.random.default_rng(args.seed).permutation(num_blocks).astype(np.int64)
    tables = [perm[b * bps:(b + 1) * bps].tolist() for b in range(B)]

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------- device-timed decode: inputs resident, tokens chained on the device
    # Each step replays the captured decode graph after one device-to-device copy of
    # that step's packed inputs (positions, context lengths, block tables), all of
    # which were uploaded before the timed region; the token ids come from the
    # previous step's argmax.
    total = W + K
    graph = DecodeGraph(model, pool, B, table_bucket(bps))
    tok0 = torch.randint(0, cfg.vocab_size, (B,), generator=torch.Generator().manual_seed(args.seed)).numpy()
    packed = []
    for i in range(total):
        buf = graph.pack(tok0, np.full(B, ctx - 1 + i, dtype=np.int64), tables,
                         np.zeros(graph.nbytes, dtype=np.uint8))
        packed.append(torch.from_numpy(buf).to(dev))
    graph.meta.copy_(packed[0])
    c0 = _lib.launch_count
    graph.capture()
    graph_launches = (_lib.launch_count - c0) // 2  # the capture runs the step eagerly once, then records it
    stream = torch.cuda.current_stream(dev)
    tok = graph.tok.clone()

    def decode_step(i, tok_in):
        graph.meta.copy_(packed[i])
        graph.tok.copy_(tok_in)
        nt, _ = graph.replay()
        return nt.view(B, 1)

    for i in range(W):
        tok = decode_step(i, tok)
    torch.cuda.synchronize(dev)
    _lib.check_device_status(dev, "warm-up")
    barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(W, total):
        tok = decode_step(i, tok)
    ev1.record(stream)
    ev1.synchronize()
    launches = graph_launches * K
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize(dev)
    _lib.check_device_status(dev, "timed decode")
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    value = B * K / (ms / 1000.0)

    # ---------------- per-kernel timing of the decode kernels (same inputs, live)
    md = graph.md  # holds the last timed step's inputs
    xn = torch.randn(B, cfg.hidden_dim, device=dev).to(model.dtype)
    kern = {}

    def time_fn(fn, reps):
        """Device time per call: `reps` calls captured in one CUDA graph, replayed 3 times."""
        fn()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for r in range(reps):
                fn(r)
        g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(3):
            g.replay()
        e1.record(stream)
        e1.synchronize()
        del g
        return e0.elapsed_time(e1) / (3 * reps) / 1000.0

    lay = model.layers
    L = len(lay)
    nq, nkv, hd = lay[0].self_attn.local_heads, lay[0].self_attn.local_kv_heads, cfg.head_dim
    q = torch.randn(B, nq * hd, device=dev).to(model.dtype)
    splits = kernels.attention_splits(B, nkv, ctx + total, 16, dev)
    attn_out = torch.empty(B, nq * hd, device=dev, dtype=model.dtype)
    scale = 1.0 / math.sqrt(hd)
    t_attn = time_fn(lambda r=0: kernels.paged_attention(q, nq, nkv, hd, pool.k_cache, pool.v_cache, r % L,
                                                         md.tables, None, md.ctx_lens, True, scale,
                                                         out=attn_out, num_splits=splits), 2 * L)
    ctx_sum = int(md.ctx_lens.sum().item())
    esz = 2
    attn_bytes = ctx_sum * nkv * hd * 2 * esz + B * nq * hd * esz * 2
    kern["paged_attention"] = {"us": t_attn * 1e6, "bytes": attn_bytes, "gbs": attn_bytes / t_attn / 1e9}

    def wbytes(w):
        return w.numel() * w.element_size()

    sa, ml = lay[0].self_attn, lay[0].mlp
    gemms = {
        "qkv": (lambda r=0: kernels.linear_qkv(xn, lay[r % L].self_attn.q_proj.packed_weight(),
                                                lay[r % L].self_attn.k_proj.packed_weight(),
                                                lay[r % L].self_attn.v_proj.packed_weight()),
                wbytes(sa.q_proj.weight) + wbytes(sa.k_proj.weight) + wbytes(sa.v_proj.weight)),
        "o_proj": (lambda r=0: kernels.linear(attn_out, lay[r % L].self_attn.out_proj.packed_weight()),
                   wbytes(sa.out_proj.weight)),
        "gate_up_swiglu": (lambda r=0: kernels.linear_swiglu(xn, lay[r % L].mlp.gate_proj.packed_weight(),
                                                             lay[r % L].mlp.up_proj.packed_weight()),
                           wbytes(ml.gate_proj.weight) + wbytes(ml.up_proj.weight)),
    }
    down_in = torch.randn(B, ml.down_proj.in_features_per_partition, device=dev).to(model.dtype)
    gemms["down"] = (lambda r=0: kernels.linear(down_in, lay[r % L].mlp.down_proj.packed_weight()),
                     wbytes(ml.down_proj.weight))
    for name, (fn, nbytes) in gemms.items():
        t = time_fn(fn, 2 * L)
        kern[name] = {"us": t * 1e6, "bytes": nbytes, "gbs": nbytes / t / 1e9}
    v0, v1 = model.vocab_slice()  # TP > 1: this rank's vocabulary rows of the lm_head
    lm_w = model.lm_head.weight[v0:v1]
    t_lm = time_fn(lambda r=0: kernels.linear(xn, lm_w, out_dtype=torch.float32), 4)
    kern["lm_head"] = {"us": t_lm * 1e6, "bytes": wbytes(lm_w), "gbs": wbytes(lm_w) / t_lm / 1e9}
    per_step = {k: v["us"] * (1 if k == "lm_head" else L) for k, v in kern.items()}
    dominant = max(per_step, key=per_step.get)
    peak, peak_kind = measured_peaks()
    dk = kern[dominant]
    roofline = {"bound": "hbm", "kernel": dominant, "achieved": dk["gbs"], "peak": peak, "unit": "GB/s",
                "frac": dk["gbs"] / peak, "peak_source": ("measured (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                                else "fallback (6.65 TB/s, an earlier copy measurement on these B200s)"),
                "traffic": (MEASURED_TRAFFIC_RATIO[dominant] * dk["bytes"]
                            if dominant in MEASURED_TRAFFIC_RATIO else None),
                "traffic_source": ("ncu capture at batch 128, context 2048, TP=1, scaled by algorithmic bytes"
                                   if dominant in MEASURED_TRAFFIC_RATIO else None),
                "algorithmic_bytes_per_launch": dk["bytes"],
                "share_of_step": per_step[dominant] / 1000.0 / (ms / K)}

    # ---------------- fused all-reduce + residual + RMSNorm bus bandwidth (TP > 1)
    fused_ar = sweep = None
    if world > 1:
        H = cfg.hidden_dim
        nw = lay[0].post_attention_layernorm.weight
        _, _, R = comm.row_slice(B)
        res = torch.zeros(R, H, device=dev)  # this rank's residual rows

        y_ar = torch.empty(B, H, device=dev, dtype=model.dtype)
        a_in = torch.randn(B, lay[0].self_attn.out_proj.in_features_per_partition, device=dev).to(model.dtype)
        w_o = lay[0].self_attn.out_proj.packed_weight()

        def ar(r=0):  # the fused row-parallel all-reduce of the decode step: GEMM push + reduce/norm/gather
            comm.row_parallel_linear(a_in, w_o)
            comm.allreduce_rmsnorm_sharded(B, H, model.dtype, res, nw, 1e-5, out=y_ar)
        # 20 back-to-back calls captured in one graph (an even count keeps the parity
        # sequence), so the number is the device time of the collective, not launch cost.
        n_ar = 20
        for _ in range(2):
            ar()
        torch.cuda.synchronize(dev)
        barrier()
        g_ar = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_ar):
            for _ in range(n_ar):
                ar()
        barrier()
        g_ar.replay()
        torch.cuda.synchronize(dev)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            g_ar.replay()
        e1.record(stream)
        e1.synchronize()
        t_ar = max_over_ranks(e0.elapsed_time(e1) / (5 * n_ar) / 1000.0)
        _lib.check_device_status(dev, "all-reduce timing")
        del g_ar
        payload = B * H * 2
        sweep = None if args.no_sweep else allreduce_sweep(comm, rank, world, dev, args.seed)
        fused_ar = {"tokens": B, "payload_bytes": payload, "us": t_ar * 1e6,
                    "bus_gbs": 2 * (world - 1) / world * payload / t_ar / 1e9,
                    "nvlink_peak_gbs": sweep["nvlink_peak_gbs"] if sweep else None,
                    "nvlink_peak_source": sweep["nvlink_peak_source"] if sweep else None,
                    "o_proj_gemm_alone_us": kern["o_proj"]["us"],
                    "note": "o_proj GEMM with the reduce-scatter pushed from its epilogue, then the "
                            "reduce + residual + RMSNorm + all-gather kernel"}

    # ---------------- end to end through WorkerExecutionEngine.execute_step
    e2e = None
    if not args.no_e2e:
        tok_host = tok.view(-1).cpu().numpy().tolist()
        pos0 = ctx - 1 + total
        steps_e2e = [None] * (W + K)
        h2d = d2h = 0

        def e2e_step(i, toks):
            slots = [SequenceSlot(seq_id=f"s{b}", is_prefill=False, current_token_id=int(toks[b]),
                                  current_len=pos0 + i + 1, block_table=tables[b]) for b in range(B)]
            resp = engine.execute_step(StepRequest(step_id=i, active_sequences=slots))
            return [t.token_id for t in resp.sampled_tokens]

        for i in range(W):
            tok_host = e2e_step(i, tok_host)
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(W, W + K):
            tok_host = e2e_step(i, tok_host)
            h2d, d2h = engine.last_h2d_bytes, engine.last_d2h_bytes
        e1.record(stream)
        e1.synchronize()
        ms_e2e = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": B * K / (ms_e2e / 1000.0), "unit": "tokens/s", "ms_per_step": ms_e2e / K,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "api": "WorkerExecutionEngine.execute_step(StepRequest) with host block tables"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline_entry(args, model_config(32))
        except Exception as e:  # pragma: no cover - reported, not fatal
            cpu = {"value": None, "unit": "tokens/s", "error": repr(e)}

    if rank == 0:
        line = {
            "metric": "decode tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: N(0,0.02) weights, random KV cache, random block-table permutation",
            "config": decode_config(args, world),
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk,
            "gpu_launches": launches, "kernels": kern, "fused_allreduce": fused_ar,
            "fused_allreduce_sweep": sweep, "parity": parity,
        }
        print(json.dumps(line), flush=True)
    if comm is not None:
        barrier()
        comm.cleanup()
    if world > 1:
        dist.destroy_process_group()
    if parity is not None and not parity["pass"]:
        print(f"parity check failed at TP={world}: {json.dumps(parity)}", file=sys.stderr)
        return 1
    return 0


# ----------------------------------------------------------------------------- prefill workload
def prefill_flops(cfg, lens, world):
    """Per rank: 2 * tokens * layer parameters + causal attention 4 * (pos + 1) * head_dim per q head."""
    H, hd, nq, nkv, inter, L = (cfg.hidden_dim, cfg.head_dim, cfg.num_heads, cfg.num_kv_heads,
                                cfg.intermediate_dim, cfg.num_layers)
    params = H * (nq + 2 * nkv) * hd + nq * hd * H + 3 * H * inter
    T = sum(lens)
    keys = sum(P * (P + 1) // 2 for P in lens)
    gemm = 2.0 * T * params * L / world
    attn = 4.0 * keys * hd * nq * L / world
    return gemm, attn


def cpu_prefill_sample(cfg, P: int, seed: int):
    """Oracle (numpy float32) prefill of one prompt of P tokens through one decoder layer; seconds."""
    import oracle
    from oracle import decoder as od
    od.set_precision(np.float32)
    rng = np.random.default_rng(seed)
    H, hd, nq, nkv, inter = cfg.hidden_dim, cfg.head_dim, cfg.num_heads, cfg.num_kv_heads, cfg.intermediate_dim
    ocfg = oracle.OracleConfig(cfg.vocab_size, H, 1, nq, nkv, inter, max(cfg.max_seq_len, P + 8), cfg.rms_norm_eps)
    std = np.float32(0.02)
    shard = {
        "layers.0.input_layernorm.weight": np.ones(H, np.float32),
        "layers.0.post_attention_layernorm.weight": np.ones(H, np.float32),
        "layers.0.self_attn.q_proj.weight": rng.standard_normal((H, nq * hd), np.float32) * std,
        "layers.0.self_attn.k_proj.weight": rng.standard_normal((H, nkv * hd), np.float32) * std,
        "layers.0.self_attn.v_proj.weight": rng.standard_normal((H, nkv * hd), np.float32) * std,
        "layers.0.self_attn.out_proj.weight": rng.standard_normal((nq * hd, H), np.float32) * std,
        "layers.0.mlp.gate_proj.weight": rng.standard_normal((H, inter), np.float32) * std,
        "layers.0.mlp.up_proj.weight": rng.standard_normal((H, inter), np.float32) * std,
        "layers.0.mlp.down_proj.weight": rng.standard_normal((inter, H), np.float32) * std,
    }
    nb = math.ceil(P / 16)
    pool = oracle.KVPool(1, nb, 16, nkv, hd)
    model = oracle.OracleModel(ocfg, [shard], [pool], cos=None, sin=None)
    h = rng.standard_normal((1, P, H), np.float32)
    pos = np.arange(P, dtype=np.int64)[None]
    t0 = time.perf_counter()
    model.block(0, h, pos, [list(range(nb))], True)
    t = time.perf_counter() - t0
    od.set_precision(np.float64)
    return t


def cpu_job_estimate(cfg, prompt_lens, dec_batch, dec_ctx, dec_steps, seed):
    """CPU time of a job of the reference's CPU path, extrapolated from bounded samples.

    Prefill: one forward per prompt (execution_engine.py:85-111), timed as one prompt of
    the mean length through 1 of the layers (the oracle's float32 prefill) and scaled by
    the layers and prompts; decode: ``dec_steps`` batched steps of ``dec_batch`` rows at
    the mean context ``dec_ctx``, each timed as 1 layer + 1/8 of the lm_head on torch CPU
    (oracle/grpc_tp.py) and extrapolated.  Returns (seconds, description)."""
    P = int(round(float(np.mean(prompt_lens)))) if len(prompt_lens) else 0
    t_pre = cpu_prefill_sample(cfg, P, seed) * cfg.num_layers * len(prompt_lens) if P else 0.0
    t_dec = 0.0
    # the restated decode holds about 64 KB of float32 K/V copies per (row, context token):
    # sample at most 131072 of them (about 8 GB) and scale by the rows
    b_s = max(1, min(dec_batch, 131072 // max(1, dec_ctx)))
    if dec_steps:
        r = cpu_decode(cfg, 1, b_s, dec_ctx, 1, 1, seed, cpu_cores())
        t_dec = statistics.median(r["step_s"]) * dec_steps * dec_batch / b_s
    desc = (f"extrapolated from samples on this host's {cpu_cores()} cores: {len(prompt_lens)} prefills as one "
            f"{P}-token prompt through 1 of {cfg.num_layers} layers (numpy float32) x prompts x layers, plus "
            f"{dec_steps} decode steps of {dec_batch} rows at context {dec_ctx}, sampled as {b_s} rows through "
            f"1 layer + 1/8 lm_head (torch CPU) x layers x {dec_batch}/{b_s}")
    return t_pre + t_dec, desc


def run_prefill(args):
    import torch
    import torch.distributed as dist

    from pythonintern_b200 import _lib, kernels, workloads
    from pythonintern_b200.config import KVCacheConfig, ShardConfig
    from pythonintern_b200.model.metadata import build_prefill_metadata
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    from pythonintern_b200.worker.execution_engine import WorkerExecutionEngine
    from pythonintern_b200.worker.messages import SequenceSlot, StepRequest

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=dev)
    cfg = workloads.mistral_7b_config(num_layers=args.layers)
    n, P, W, K = args.prompts, args.prompt_len, args.warmup, args.steps
    lens = [P] * n
    T = sum(lens)
    comm = None
    if world > 1:
        comm = DistributedCommunicator(rank, world, device=dev, max_bytes=max(64 << 20, T * cfg.hidden_dim * 2))
        comm.connect()
    bps = math.ceil(P / 16)
    num_blocks = n * bps + 8
    engine = WorkerExecutionEngine(cfg, ShardConfig(rank=rank, world_size=world),
                                   KVCacheConfig(block_size=16, num_blocks=num_blocks, device=str(dev)), comm, dev,
                                   max_prefill_tokens=T)
    model, pool = engine.model, engine.kv_manager.pool
    init_synthetic(model, pool, args.seed, rank, dev)
    perm = np.random.default_rng(args.seed).permutation(num_blocks).astype(np.int64)
    tables = [perm[s * bps:(s + 1) * bps].tolist() for s in range(n)]
    prompts = np.random.default_rng(args.seed + 7).integers(0, cfg.vocab_size, size=(n, P)).astype(np.int64)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------- device-timed: prompts and metadata resident in HBM
    md = build_prefill_metadata(lens, tables, dev)
    ids = torch.from_numpy(prompts.reshape(1, T)).to(dev)

    def step(i):
        return model.greedy(ids, None, pool, tables, True, i, metadata=md)

    for i in range(W):
        step(i)
    torch.cuda.synchronize(dev)
    _lib.check_device_status(dev, "prefill warm-up")
    barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    c0 = _lib.launch_count
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(W, W + K):
        step(i)
    ev1.record(stream)
    ev1.synchronize()
    launches = _lib.launch_count - c0
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize(dev)
    _lib.check_device_status(dev, "timed prefill")
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    value = T * K / (ms / 1000.0)

    # ---------------- per-kernel device time at the same token count
    lay = model.layers
    L = len(lay)
    sa, ml = lay[0].self_attn, lay[0].mlp
    nq, nkv, hd = sa.local_heads, sa.local_kv_heads, cfg.head_dim
    H = cfg.hidden_dim
    xn = torch.randn(T, H, device=dev).to(model.dtype)
    q = torch.randn(T, nq * hd, device=dev).to(model.dtype)
    attn_out = torch.empty(T, nq * hd, device=dev, dtype=model.dtype)
    inter_in = torch.randn(T, ml.down_proj.in_features_per_partition, device=dev).to(model.dtype)

    def time_calls(fn, reps):
        fn(0)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for r in range(reps):
            fn(r)
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps / 1000.0

    gemm_f = {"qkv": 2.0 * T * H * (nq + 2 * nkv) * hd, "o_proj": 2.0 * T * nq * hd * H,
              "gate_up_swiglu": 2.0 * T * H * 2 * ml.down_proj.in_features_per_partition,
              "down": 2.0 * T * ml.down_proj.in_features_per_partition * H}
    fns = {
        "qkv": lambda r: kernels.linear_qkv(xn, lay[r % L].self_attn.q_proj.packed_weight(),
                                            lay[r % L].self_attn.k_proj.packed_weight(),
                                            lay[r % L].self_attn.v_proj.packed_weight()),
        "prefill_attention": lambda r: kernels.prefill_attention(q, nq, nkv, hd, pool.k_cache, pool.v_cache, r % L,
                                                                 md.tables, md.seq_start, md.n_seqs,
                                                                 1.0 / math.sqrt(hd), out=attn_out),
        "o_proj": lambda r: kernels.linear(attn_out, lay[r % L].self_attn.out_proj.packed_weight()),
        "gate_up_swiglu": lambda r: kernels.linear_swiglu(xn, lay[r % L].mlp.gate_proj.packed_weight(),
                                                          lay[r % L].mlp.up_proj.packed_weight()),
        "down": lambda r: kernels.linear(inter_in, lay[r % L].mlp.down_proj.packed_weight()),
    }
    attn_f = 4.0 * sum(p * (p + 1) // 2 for p in lens) * hd * nq
    kern = {}
    for name, fn in fns.items():
        t = time_calls(fn, 4)
        f = attn_f if name == "prefill_attention" else gemm_f[name]
        kern[name] = {"us": t * 1e6, "flops": f, "tflops": f / t / 1e12}
    torch.cuda.synchronize(dev)
    _lib.check_device_status(dev, "prefill kernel timing")
    per_step = {k: v["us"] * L for k, v in kern.items()}
    dominant = max(per_step, key=per_step.get)
    peak, peak_kind = measured_tensor_peak()
    dk = kern[dominant]
    g_fl, a_fl = prefill_flops(cfg, lens, world)
    roofline = {"bound": "tensor", "kernel": dominant, "achieved": dk["tflops"], "peak": peak, "unit": "TFLOP/s",
                "frac": dk["tflops"] / peak,
                "peak_source": ("measured (MEASURED_PEAKS.json bf16_tflops)" if peak_kind == "measured"
                                else "fallback (1.59 PFLOP/s, an earlier cuBLAS bf16 measurement on these B200s)"),
                "traffic": None, "algorithmic_flops_per_launch": dk["flops"],
                "share_of_step": per_step[dominant] / 1000.0 / (ms / K),
                "step_tflops": (g_fl + a_fl) / (ms / K / 1000.0) / 1e12}

    # ---------------- end to end: StepRequests with host prompts through execute_step
    e2e = None
    if not args.no_e2e:
        h2d = d2h = 0

        def e2e_step(i):
            slots = [SequenceSlot(seq_id=f"p{s}", is_prefill=True, prompt_token_ids=prompts[s].tolist(),
                                  current_len=P, block_table=tables[s]) for s in range(n)]
            engine.execute_step(StepRequest(step_id=i, active_sequences=slots))

        for i in range(W):
            e2e_step(i)
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(W, W + K):
            e2e_step(i)
            h2d, d2h = engine.last_h2d_bytes, engine.last_d2h_bytes
        e1.record(stream)
        e1.synchronize()
        ms_e2e = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": T * K / (ms_e2e / 1000.0), "unit": "tokens/s", "ms_per_step": ms_e2e / K,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "api": "WorkerExecutionEngine.execute_step(StepRequest) with host prompts"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            t1 = cpu_prefill_sample(cfg, P, args.seed)
            step_s = t1 * cfg.num_layers * n
            cpu = {"value": T / step_s, "unit": "tokens/s", "cores": cpu_cores(), "kind": "port",
                   "sample": (f"oracle (numpy float32 restatement of the reference CPU path): one prompt of {P} "
                              f"tokens through 1 of {cfg.num_layers} decoder layers, extrapolated to "
                              f"{n} prompts x {cfg.num_layers} layers (the reference prefills one prompt per forward)")}
        except Exception as e:  # pragma: no cover - reported, not fatal
            cpu = {"value": None, "unit": "tokens/s", "error": repr(e)}

    if rank == 0:
        line = {
            "metric": "prefill tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: N(0,0.02) weights, random prompts, random block-table permutation",
            "config": {"workload": (f"mistral-7b-shape batched prefill, {n} prompts x {P} tokens, TP={world}"
                                    f" ({cfg.num_layers} layers)"),
                       "model": "mistral-7b-shape", "global_batch": n, "seq_len": P, "parallelism": f"tp{world}",
                       "l2": "inputs larger than L2 (weights read per step >> 126 MB)"},
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk,
            "gpu_launches": launches, "kernels": kern,
        }
        print(json.dumps(line), flush=True)
    if comm is not None:
        barrier()
        comm.cleanup()
    if world > 1:
        dist.destroy_process_group()
    return 0


# ----------------------------------------------------------------------------- mixed continuous-batching step
MIXED_PREFILLS, MIXED_PROMPT, MIXED_DECODES, MIXED_CTX = 16, 1024, 240, (512, 8192)


def mixed_layout(seed: int):
    """One mixed step's sequences: 16 prompts of 1024 tokens and 240 decodes whose contexts are
    uniform in [512, 8192] (seeded); every sequence's blocks from one seeded permutation."""
    rng = np.random.default_rng(seed + 11)
    dec_ctx = rng.integers(MIXED_CTX[0], MIXED_CTX[1] + 1, size=MIXED_DECODES).astype(np.int64)
    nblk_p = math.ceil(MIXED_PROMPT / 16)
    nblk_d = [math.ceil(int(c) / 16) for c in dec_ctx]
    total = MIXED_PREFILLS * nblk_p + sum(nblk_d) + 8
    perm = rng.permutation(total).astype(np.int64)
    k, tp, td = 0, [], []
    for _ in range(MIXED_PREFILLS):
        tp.append(perm[k:k + nblk_p].tolist())
        k += nblk_p
    for n in nblk_d:
        td.append(perm[k:k + n].tolist())
        k += n
    prompts = rng.integers(0, 32000, size=(MIXED_PREFILLS, MIXED_PROMPT)).astype(np.int64)
    dec_tok = rng.integers(0, 32000, size=MIXED_DECODES).astype(np.int64)
    return prompts, tp, dec_ctx, dec_tok, td, total


def run_mixed(args):
    """Config 4: one continuous-batching step of the Mistral-7B shape (vocab 32000) holding 16
    prefills of 1024 tokens and 240 decodes at contexts uniform in [512, 8192], tensor parallel
    over the ranks.  The reference runs the prefills one forward each and then the decodes as
    one batch (engine/worker/execution_engine.py:85-145); here the step is one varlen prefill
    forward plus one replay of the captured decode step.  Metric: tokens processed per second
    (prompt tokens + decode tokens) by the step."""
    import torch
    import torch.distributed as dist

    from pythonintern_b200 import _lib, workloads
    from pythonintern_b200.config import KVCacheConfig, ShardConfig
    from pythonintern_b200.model.metadata import build_prefill_metadata
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    from pythonintern_b200.worker.execution_engine import WorkerExecutionEngine
    from pythonintern_b200.worker.graphs import DecodeGraph, table_bucket
    from pythonintern_b200.worker.messages import SequenceSlot, StepRequest

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=180), device_id=dev)
    cfg = workloads.mistral_7b_config(num_layers=args.layers, max_seq_len=8448)
    W, K = args.warmup, args.steps
    prompts, tp, dec_ctx, dec_tok, td, num_blocks = mixed_layout(args.seed)
    T_p = MIXED_PREFILLS * MIXED_PROMPT
    comm = None
    if world > 1:
        comm = DistributedCommunicator(rank, world, device=dev, max_bytes=T_p * cfg.hidden_dim * 2)
        comm.connect()
    engine = WorkerExecutionEngine(cfg, ShardConfig(rank=rank, world_size=world),
                                   KVCacheConfig(block_size=16, num_blocks=num_blocks, device=str(dev)), comm, dev,
                                   max_prefill_tokens=T_p)
    model, pool = engine.model, engine.kv_manager.pool
    init_synthetic(model, pool, args.seed, rank, dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------- device-timed: the step's inputs resident in HBM
    md_p = build_prefill_metadata([MIXED_PROMPT] * MIXED_PREFILLS, tp, dev)
    ids_p = torch.from_numpy(prompts.reshape(1, T_p)).to(dev)
    graph = DecodeGraph(model, pool, MIXED_DECODES, table_bucket(max(len(t) for t in td)))
    graph.meta.copy_(torch.from_numpy(graph.pack(dec_tok, dec_ctx - 1, td, np.zeros(graph.nbytes, np.uint8))).to(dev))
    c0 = _lib.launch_count
    graph.capture()
    dec_launches = (_lib.launch_count - c0) // 2

    def prefill(i):
        return model.greedy(ids_p, None, pool, tp, True, i, metadata=md_p)

    def step(i):
        prefill(i)
        return graph.replay()

    for i in range(W):
        step(i)
    torch.cuda.synchronize(dev)
    _lib.check_device_status(dev, "mixed warm-up")
    barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    c1 = _lib.launch_count
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(W, W + K):
        step(i)
    ev1.record(stream)
    ev1.synchronize()
    clk = clocks.stop()
    launches = (_lib.launch_count - c1) + dec_launches * K
    barrier()
    torch.cuda.synchronize(dev)
    _lib.check_device_status(dev, "timed mixed step")
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    tokens = T_p + MIXED_DECODES
    value = tokens * K / (ms / 1000.0)

    # ---------------- the two halves timed apart (same inputs)
    def time_part(fn, reps=3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for r in range(reps):
            fn(r)
        e1.record(stream)
        e1.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / reps)
    ms_pre = time_part(prefill)
    ms_dec = time_part(lambda r: graph.replay())
    g_fl, a_fl = prefill_flops(cfg, [MIXED_PROMPT] * MIXED_PREFILLS, world)
    H, hd, nkv, L = cfg.hidden_dim, cfg.head_dim, cfg.num_kv_heads, cfg.num_layers
    wbytes = L * (H * (cfg.num_heads + 2 * nkv) * hd + cfg.num_heads * hd * H + 3 * H * cfg.intermediate_dim) * 2
    kv_bytes = L * int(dec_ctx.sum()) * 2 * nkv * hd * 2
    dec_bytes = (wbytes + kv_bytes) / world + cfg.vocab_size * H * 2 / world
    t_peak, t_kind = measured_tensor_peak()
    h_peak, h_kind = measured_peaks()
    pre_tf = (g_fl + a_fl) / (ms_pre / 1000.0) / 1e12
    dec_gbs = dec_bytes / (ms_dec / 1000.0) / 1e9
    roofline = {"bound": "tensor", "kernel": "prefill half of the step (all its GEMMs and attention)",
                "achieved": pre_tf, "peak": t_peak, "unit": "TFLOP/s", "frac": pre_tf / t_peak,
                "peak_source": f"{t_kind} (bf16_tflops)", "traffic": None,
                "share_of_step": ms_pre / (ms / K),
                "decode_half": {"ms": ms_dec, "algorithmic_bytes": dec_bytes, "gbs": dec_gbs, "peak_gbs": h_peak,
                                "frac": dec_gbs / h_peak, "peak_source": f"{h_kind} (hbm_gbs)"}}

    # ---------------- end to end through execute_step: host prompts, tables and tokens
    e2e = None
    if not args.no_e2e:
        h2d = d2h = 0

        def e2e_step(i):
            slots = [SequenceSlot(seq_id=f"p{s}", is_prefill=True, prompt_token_ids=prompts[s].tolist(),
                                  current_len=MIXED_PROMPT, block_table=tp[s]) for s in range(MIXED_PREFILLS)]
            slots += [SequenceSlot(seq_id=f"d{d}", is_prefill=False, current_token_id=int(dec_tok[d]),
                                   current_len=int(dec_ctx[d]), block_table=td[d]) for d in range(MIXED_DECODES)]
            engine.execute_step(StepRequest(step_id=i, active_sequences=slots))

        for i in range(W):
            e2e_step(i)
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(W, W + K):
            e2e_step(i)
            h2d, d2h = engine.last_h2d_bytes, engine.last_d2h_bytes
        e1.record(stream)
        e1.synchronize()
        ms_e2e = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": tokens * K / (ms_e2e / 1000.0), "unit": "tokens/s", "ms_per_step": ms_e2e / K,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "api": "WorkerExecutionEngine.execute_step(StepRequest) with 16 prefill + 240 decode slots"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            t_cpu, desc = cpu_job_estimate(cfg, [MIXED_PROMPT] * MIXED_PREFILLS, MIXED_DECODES,
                                           int(dec_ctx.mean()), 1, args.seed)
            cpu = {"value": tokens / t_cpu, "unit": "tokens/s", "cores": cpu_cores(), "kind": "port",
                   "sample": desc}
        except Exception as e:  # pragma: no cover - reported, not fatal
            cpu = {"value": None, "unit": "tokens/s", "error": repr(e)}
    if rank == 0:
        line = {
            "metric": "mixed-step tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: N(0,0.02) weights, random KV cache and prompts, random block-table permutation",
            "config": {"workload": (f"mistral-7b-shape mixed step: {MIXED_PREFILLS} prefills x {MIXED_PROMPT} tokens "
                                    f"+ {MIXED_DECODES} decodes at contexts uniform {MIXED_CTX[0]}-{MIXED_CTX[1]}, "
                                    f"TP={world} ({cfg.num_layers} layers)"),
                       "model": "mistral-7b-shape", "global_batch": MIXED_PREFILLS + MIXED_DECODES,
                       "seq_len": MIXED_PROMPT, "parallelism": f"tp{world}",
                       "l2": "inputs larger than L2 (weights + KV read per step >> 126 MB)"},
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk, "gpu_launches": launches,
            "parts_ms": {"prefill": ms_pre, "decode": ms_dec},
        }
        print(json.dumps(line), flush=True)
    del graph
    if comm is not None:
        barrier()
        comm.cleanup()
    if world > 1:
        dist.destroy_process_group()
    return 0


# ----------------------------------------------------------------------------- continuous batching, TinyLlama
TL_REQUESTS, TL_PROMPT, TL_NEW = 64, (128, 512), 128


def tinyllama_job(seed: int):
    """64 requests with prompts uniform in [128, 512] tokens (seeded), 128 new tokens each; block
    tables cover prompt + new tokens, all slices of one seeded permutation of the pool."""
    rng = np.random.default_rng(seed + 23)
    lens = rng.integers(TL_PROMPT[0], TL_PROMPT[1] + 1, size=TL_REQUESTS).astype(np.int64)
    prompts = [rng.integers(0, 32000, size=int(n)).astype(np.int64) for n in lens]
    nblk = [math.ceil((int(n) + TL_NEW) / 16) for n in lens]
    total = sum(nblk) + 8
    perm = rng.permutation(total).astype(np.int64)
    tables, k = [], 0
    for n in nblk:
        tables.append(perm[k:k + n].tolist())
        k += n
    return prompts, lens, tables, total


def run_tinyllama(args):
    """Config 2: TinyLlama 1.1B shape (bf16), 64 requests admitted together (continuous batching
    with max_batch_size >= 64, so the batcher's first step prefills them all and every later
    step decodes all 64, engine/scheduler/continuous_batcher.py:53-108), 128 greedy tokens each,
    tensor parallel over the ranks.  One bench step = the whole job (1 prefill step + 127
    decode steps); metric = generated tokens per second."""
    import torch
    import torch.distributed as dist

    from pythonintern_b200 import _lib, workloads
    from pythonintern_b200.config import KVCacheConfig, ShardConfig
    from pythonintern_b200.model.metadata import build_prefill_metadata
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    from pythonintern_b200.worker.execution_engine import WorkerExecutionEngine
    from pythonintern_b200.worker.graphs import DecodeGraph, table_bucket
    from pythonintern_b200.worker.messages import SequenceSlot, StepRequest

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=180), device_id=dev)
    cfg = workloads.tinyllama_config(num_layers=22 if args.layers == 32 else args.layers)
    cfg.max_seq_len = 1024
    W, K = args.warmup, args.steps
    prompts, lens, tables, num_blocks = tinyllama_job(args.seed)
    T_p = int(lens.sum())
    comm = None
    if world > 1:
        comm = DistributedCommunicator(rank, world, device=dev, max_bytes=T_p * cfg.hidden_dim * 2)
        comm.connect()
    engine = WorkerExecutionEngine(cfg, ShardConfig(rank=rank, world_size=world),
                                   KVCacheConfig(block_size=16, num_blocks=num_blocks, device=str(dev)), comm, dev,
                                   max_prefill_tokens=T_p)
    model, pool = engine.model, engine.kv_manager.pool
    init_synthetic(model, pool, args.seed, rank, dev)
    stream = torch.cuda.current_stream(dev)
    B = TL_REQUESTS

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------- device-timed job: prompts, tables and every decode step's metadata resident
    md_p = build_prefill_metadata(lens.tolist(), tables, dev)
    ids_p = torch.from_numpy(np.concatenate(prompts)[None]).to(dev)
    graph = DecodeGraph(model, pool, B, table_bucket(max(len(t) for t in tables)))
    packed = []
    for i in range(1, TL_NEW):
        buf = graph.pack(np.zeros(B, np.int64), lens - 1 + i, tables, np.zeros(graph.nbytes, np.uint8))
        packed.append(torch.from_numpy(buf).to(dev))
    graph.meta.copy_(packed[0])
    c0 = _lib.launch_count
    graph.capture()
    dec_launches = (_lib.launch_count - c0) // 2
    out_tok = torch.empty(TL_NEW, B, dtype=torch.int64, device=dev)

    def job():
        tok, _ = model.greedy(ids_p, None, pool, tables, True, 0, metadata=md_p)
        out_tok[0].copy_(tok.view(-1))
        for i in range(1, TL_NEW):
            graph.meta.copy_(packed[i - 1])
            graph.tok.copy_(out_tok[i - 1].view(B, 1))
            nt, _ = graph.replay()
            out_tok[i].copy_(nt.view(-1))

    for _ in range(W):
        job()
    torch.cuda.synchronize(dev)
    _lib.check_device_status(dev, "tinyllama warm-up")
    barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    c1 = _lib.launch_count
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(K):
        job()
    ev1.record(stream)
    ev1.synchronize()
    clk = clocks.stop()
    launches = (_lib.launch_count - c1) + dec_launches * (TL_NEW - 1) * K
    barrier()
    torch.cuda.synchronize(dev)
    _lib.check_device_status(dev, "timed tinyllama job")
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    gen = B * TL_NEW
    value = gen * K / (ms / 1000.0)

    # decode steps alone: HBM roofline of the decode step (weights + KV read per step)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for i in range(1, TL_NEW):
        graph.meta.copy_(packed[i - 1])
        graph.replay()
    e1.record(stream)
    e1.synchronize()
    ms_dec = max_over_ranks(e0.elapsed_time(e1)) / (TL_NEW - 1)
    H, hd, nkv, L = cfg.hidden_dim, cfg.head_dim, cfg.num_kv_heads, cfg.num_layers
    wbytes = L * (H * (cfg.num_heads + 2 * nkv) * hd + cfg.num_heads * hd * H + 3 * H * cfg.intermediate_dim) * 2
    kv_avg = float(lens.mean()) + TL_NEW / 2
    dec_bytes = (wbytes + L * B * kv_avg * 2 * nkv * hd * 2) / world + cfg.vocab_size * H * 2 / world
    peak, kind = measured_peaks()
    gbs = dec_bytes / (ms_dec / 1000.0) / 1e9
    roofline = {"bound": "hbm", "kernel": "decode step (captured graph), weights + KV per step", "achieved": gbs,
                "peak": peak, "unit": "GB/s", "frac": gbs / peak, "peak_source": f"{kind} (hbm_gbs)", "traffic": None,
                "algorithmic_bytes_per_step": dec_bytes, "decode_step_ms": ms_dec,
                "share_of_job": ms_dec * (TL_NEW - 1) / (ms / K)}

    # ---------------- end to end: the job through execute_step with a host-side batcher
    e2e = None
    if not args.no_e2e:
        h2d = d2h = 0

        def e2e_job():
            nonlocal h2d, d2h
            slots = [SequenceSlot(seq_id=f"r{r}", is_prefill=True, prompt_token_ids=prompts[r].tolist(),
                                  current_len=int(lens[r]), block_table=tables[r]) for r in range(B)]
            resp = engine.execute_step(StepRequest(step_id=0, active_sequences=slots))
            h2d, d2h = engine.last_h2d_bytes, engine.last_d2h_bytes
            cur = {t.seq_id: t.token_id for t in resp.sampled_tokens}
            for i in range(1, TL_NEW):
                slots = [SequenceSlot(seq_id=f"r{r}", is_prefill=False, current_token_id=cur[f"r{r}"],
                                      current_len=int(lens[r]) + i, block_table=tables[r]) for r in range(B)]
                resp = engine.execute_step(StepRequest(step_id=i, active_sequences=slots))
                cur = {t.seq_id: t.token_id for t in resp.sampled_tokens}
                h2d += engine.last_h2d_bytes
                d2h += engine.last_d2h_bytes

        for _ in range(W):
            e2e_job()
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(K):
            e2e_job()
        e1.record(stream)
        e1.synchronize()
        ms_e2e = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": gen * K / (ms_e2e / 1000.0), "unit": "tokens/s", "ms_per_step": ms_e2e / K,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "api": "WorkerExecutionEngine.execute_step: 1 prefill step of 64 prompts + 127 decode steps"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            t_cpu, desc = cpu_job_estimate(cfg, lens.tolist(), B, int(lens.mean()) + TL_NEW // 2, TL_NEW - 1,
                                           args.seed)
            cpu = {"value": gen / t_cpu, "unit": "tokens/s", "cores": cpu_cores(), "kind": "port", "sample": desc}
        except Exception as e:  # pragma: no cover - reported, not fatal
            cpu = {"value": None, "unit": "tokens/s", "error": repr(e)}
    if rank == 0:
        line = {
            "metric": "generated tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: N(0,0.02) weights, random prompts, random block-table permutation",
            "config": {"workload": (f"tinyllama-1.1b-shape continuous batching: {B} requests, prompts uniform "
                                    f"{TL_PROMPT[0]}-{TL_PROMPT[1]} tokens, {TL_NEW} greedy tokens each, one step = "
                                    f"the whole job, TP={world} ({cfg.num_layers} layers)"),
                       "model": "tinyllama-1.1b-shape", "global_batch": B, "seq_len": TL_PROMPT[1] + TL_NEW,
                       "parallelism": f"tp{world}",
                       "l2": "inputs larger than L2 (2.2 GB of weights read per decode step)"},
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk, "gpu_launches": launches,
            "prompt_tokens_per_job": T_p,
        }
        print(json.dumps(line), flush=True)
    del graph
    if comm is not None:
        barrier()
        comm.cleanup()
    if world > 1:
        dist.destroy_process_group()
    return 0


# ----------------------------------------------------------------------------- row-parallel all-reduce
def run_allreduce(args):
    import torch
    import torch.distributed as dist

    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2:
        print(json.dumps({"metric": "row-parallel all-reduce bus GB/s", "unavailable":
                          "needs >= 2 ranks (torchrun --nproc-per-node N)"}), flush=True)
        return 0
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    comm = DistributedCommunicator(rank, world, device=dev, max_bytes=64 << 20)
    comm.connect()
    clocks = ClockSampler(local)
    clocks.start()
    sweep = allreduce_sweep(comm, rank, world, dev, args.seed)
    clk = clocks.stop()
    if rank == 0:
        top = sweep["sizes"][-1]
        line = {
            "metric": "row-parallel all-reduce bus GB/s", "value": top["fused_bus_gbs"], "unit": "GB/s",
            "n_gpus": world, "steps": None, "warmup": 2, "ms_per_step": top["fused_us"] / 1000.0,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) activations, N(0,0.02) weights",
            "config": rowpar_config(world), "clocks": clk, **sweep,
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    comm.cleanup()
    dist.destroy_process_group()
    return 0


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "prefill":
        return run_prefill(args)
    if args.workload == "allreduce":
        return run_allreduce(args)
    if args.workload == "mixed":
        return run_mixed(args)
    if args.workload == "tinyllama":
        return run_tinyllama(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
