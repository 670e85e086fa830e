#!/usr/bin/env python
"""Decode throughput of the tensor-parallel decoder-layer forward on B200.

Workload (default): the Llama-3-8B shape (hidden 4096, 32 layers, 32 q / 8 kv heads,
intermediate 14336, vocab 128256), bf16, decoding a batch of 128 sequences at
context 2048 in the paged KV cache (block_size 16, block tables a seeded random
permutation of the pool), tensor parallel over N GPUs (one process per GPU; the
row-parallel all-reduce runs over NVLink peer memory).  Weights are N(0, 0.02)
and the KV cache is random (synthetic data; there is no checkpoint or dataset).

  python bench.py --gpus N --steps K --warmup W           # this framework
  python bench.py --impl reference --steps K --warmup W   # reference CPU algorithm
  python bench.py --workload prefill                      # batched varlen prefill (below)
  torchrun --nproc-per-node N bench.py --workload allreduce   # row-parallel all-reduce (below)

One JSON line on rank 0:
  value        decode tokens/s with inputs resident in HBM (CUDA events, max over ranks)
  e2e          the same through WorkerExecutionEngine.execute_step with host-side
               StepRequests: pinned H2D of the step's inputs and D2H of the sampled
               tokens and top logits inside the timed region
  roofline     the dominant kernel's achieved HBM GB/s vs the measured copy peak
  cpu_baseline the oracle restatement of the reference's CPU path on this host's
               cores, on a bounded sample (one decoder layer of a few sequences),
               extrapolated to a full step

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
    ap.add_argument("--cpu-sample-batch", type=int, default=4)
    ap.add_argument("--workload", choices=["decode", "prefill", "allreduce"], default="decode")
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
    """nvidia-smi clocks and throttle reasons, sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="b2clk", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
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
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU leg
def cpu_sample(cfg, batch: int, ctx: int, seed: int, reps: int = 1):
    """Oracle (numpy float32) timing of one decoder layer + an lm_head slice; returns step seconds.

    The sample decodes ``batch`` sequences at context ``ctx`` through one decoder layer
    of the configured shape (the reference's per-sequence gather, zero padding,
    repeat_kv and float32 arithmetic, restated in oracle/), and multiplies the
    final hidden states by a 1/8 slice of the lm_head; the step time is
    layer_time * num_layers + slice_time * 8.
    """
    import oracle
    from oracle import decoder as od
    od.set_precision(np.float32)
    rng = np.random.default_rng(seed)
    H, hd, nq, nkv, inter = cfg.hidden_dim, cfg.head_dim, cfg.num_heads, cfg.num_kv_heads, cfg.intermediate_dim
    ocfg = oracle.OracleConfig(cfg.vocab_size, H, 1, nq, nkv, inter, max(cfg.max_seq_len, ctx + 8), cfg.rms_norm_eps)
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
    bps = math.ceil((ctx + 1) / 16)
    pool = oracle.KVPool(1, batch * bps, 16, nkv, hd)
    pool.k[:] = rng.standard_normal(pool.k.shape, np.float32)
    pool.v[:] = rng.standard_normal(pool.v.shape, np.float32)
    perm = rng.permutation(batch * bps)
    tables = [list(perm[b * bps:(b + 1) * bps]) for b in range(batch)]
    model = oracle.OracleModel(ocfg, [shard], [pool], cos=None, sin=None)
    h = rng.standard_normal((batch, 1, H), np.float32)
    pos = np.full((batch, 1), ctx - 1, dtype=np.int64)
    vs = cfg.vocab_size // 8
    lm = rng.standard_normal((vs, H), np.float32) * std
    best = None
    for _ in range(reps):
        t0 = time.perf_counter()
        y = model.block(0, h, pos, tables, False)
        t1 = time.perf_counter()
        od.rmsnorm(y[:, -1], np.ones(H, np.float32), 1e-5) @ lm.T
        t2 = time.perf_counter()
        step = (t1 - t0) * cfg.num_layers + (t2 - t1) * (cfg.vocab_size / vs)
        best = step if best is None else min(best, step)
    od.set_precision(np.float64)
    return best


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline_entry(args, cfg):
    b = max(1, min(args.cpu_sample_batch, args.batch))
    t = cpu_sample(cfg, b, args.ctx, args.seed)
    return {"value": b / t, "unit": "tokens/s", "cores": cpu_cores(), "kind": "port",
            "sample": (f"oracle (numpy float32 restatement of the reference CPU path) on {b} sequences at "
                       f"context {args.ctx}: 1 of {cfg.num_layers} decoder layers + 1/8 of the lm_head, "
                       f"extrapolated to a full decode step; TP=1 on the host cores")}


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
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if args.workload == "prefill":
        return run_reference_prefill(args)
    if args.workload == "allreduce":
        print(json.dumps({"impl": "reference", "metric": "row-parallel all-reduce bus GB/s",
                          "unavailable": "the reference all-reduce runs over gRPC between worker processes; "
                                         "it has no device path to time on these GPUs"}), flush=True)
        return 0
    cfg = model_config(32)
    b = max(1, min(args.cpu_sample_batch, args.batch))
    for _ in range(max(0, args.warmup)):
        cpu_sample(cfg, b, args.ctx, args.seed)
    times = [cpu_sample(cfg, b, args.ctx, args.seed) for _ in range(max(1, args.steps))]
    t = statistics.median(times)
    value = b / t
    line = {
        "impl": "reference", "metric": "decode tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1000.0,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": workload_name(args, 1), "model": "llama3-8b-shape",
                                        "global_batch": args.batch, "seq_len": args.ctx, "parallelism": "tp1 (CPU)"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cpu_cores(), "kind": "port",
                         "sample": f"per step: 1 of 32 decoder layers + 1/8 lm_head on {b} sequences at "
                                   f"context {args.ctx}, extrapolated; median of {len(times)} steps"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


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
        comm = DistributedCommunicator(rank, world, device=dev, max_bytes=max(1 << 24, B * cfg.hidden_dim * 2 * 2))
        comm.connect()
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
    fused_ar = None
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
        fused_ar = {"tokens": B, "payload_bytes": payload, "us": t_ar * 1e6,
                    "bus_gbs": 2 * (world - 1) / world * payload / t_ar / 1e9,
                    "nvlink_peak_gbs_per_direction": 770.0,
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
            "config": {"workload": workload_name(args, world), "model": "llama3-8b-shape", "global_batch": B,
                       "seq_len": ctx, "parallelism": f"tp{world}",
                       "l2": "inputs larger than L2 (weights + KV read per step >> 126 MB)"},
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk,
            "gpu_launches": launches, "kernels": kern, "fused_allreduce": fused_ar,
        }
        print(json.dumps(line), flush=True)
    if comm is not None:
        barrier()
        comm.cleanup()
    if world > 1:
        dist.destroy_process_group()
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


# ----------------------------------------------------------------------------- row-parallel all-reduce
def run_allreduce(args):
    import torch
    import torch.distributed as dist

    from pythonintern_b200 import _lib, kernels
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
    H, I = 4096, 14336
    Tmax = 4096
    K = I // world
    comm = DistributedCommunicator(rank, world, device=dev, max_bytes=max(64 << 20, Tmax * H * 2))
    comm.connect()
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed + 1 + rank)
    w = (torch.randn(H, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)  # packed [out, in] rows
    nw = torch.ones(H, device=dev)
    stream = torch.cuda.current_stream(dev)

    def max_over_ranks(x: float) -> float:
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def time_graph(fn, n, reps=5):
        """Device seconds per call: n calls captured in one graph, replayed `reps` times, max over ranks."""
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

    rows = []
    clocks = ClockSampler(local)
    clocks.start()
    for T in (1, 8, 64, 512, 4096):
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
        payload = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
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
        t_nccl = max_over_ranks(e0.elapsed_time(e1) / n / 1000.0)
        nbytes = T * H * 2
        bus = 2 * (world - 1) / world * nbytes
        rows.append({"tokens": T, "payload_bytes": nbytes, "fused_us": t_fused * 1e6, "gemm_alone_us": t_gemm * 1e6,
                     "fused_bus_gbs": bus / t_fused / 1e9, "nccl_allreduce_us": t_nccl * 1e6,
                     "nccl_bus_gbs": bus / t_nccl / 1e9,
                     "gemm_plus_nccl_us": (t_gemm + t_nccl) * 1e6})
    clk = clocks.stop()
    _lib.check_device_status(dev, "all-reduce microbenchmark")
    if rank == 0:
        top = rows[-1]
        line = {
            "metric": "row-parallel all-reduce bus GB/s", "value": top["fused_bus_gbs"], "unit": "GB/s",
            "n_gpus": world, "steps": None, "warmup": 2, "ms_per_step": top["fused_us"] / 1000.0,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) activations, N(0,0.02) weights",
            "config": {"workload": (f"row-parallel GEMM [T, {I}/{world}] x [{I}/{world}, {H}] + all-reduce + residual "
                                    f"+ RMSNorm, TP={world}; value at T=4096"),
                       "parallelism": f"tp{world}", "tokens": [r["tokens"] for r in rows]},
            "nvlink_peak_gbs_per_direction": 770.0,
            "note": ("fused_us includes the GEMM (its epilogue pushes the partial rows); bus GB/s counts the "
                     "all-reduce payload only, so the GEMM's time lowers it; gemm_plus_nccl_us is the unfused "
                     "alternative (GEMM, then an NCCL all-reduce, without the residual and RMSNorm)"),
            "clocks": clk, "sizes": rows,
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
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
