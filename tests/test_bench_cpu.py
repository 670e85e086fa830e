"""The CPU legs of bench.py (the reference-algorithm arm) run without a GPU."""

import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_cpu_decode_small_shape_tp1_and_tp2():
    """The reference-arm timing at a small shape: one rank, then two rank processes over gRPC."""
    import bench
    from pythonintern_b200 import workloads
    cfg = workloads.tinyllama_config(num_layers=2)
    cfg.vocab_size = 1024
    for world in (1, 2):
        r = bench.cpu_decode(cfg, world, batch=2, ctx=64, steps=2, warmup=1, seed=0, cores=2)
        assert len(r["step_s"]) == 2 and all(0 < t < 60 for t in r["step_s"])
        assert r["threads_used"] == [max(1, 2 // world)] * world


def test_reference_arm_prints_one_json_line():
    env = dict(os.environ, RANK="0", WORLD_SIZE="1")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--batch", "2", "--ctx", "64"],
                         capture_output=True, text=True, timeout=600, env=env)
    assert out.returncode == 0, out.stderr
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["cpu_baseline"]["batch"] == 2 and d["cpu_baseline"]["layers_sampled"] == 1
    assert d["config"]["parallelism"] == "tp1" and d["config"]["global_batch"] == 2


def test_reference_arm_other_ranks_exit_quietly():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2"],
                         capture_output=True, text=True, timeout=120, env=env)
    assert out.returncode == 0 and out.stdout.strip() == ""


def test_cpu_prefill_sample_and_flop_count():
    import bench
    from pythonintern_b200 import workloads
    cfg = workloads.tinyllama_config(num_layers=2)
    cfg.vocab_size = 1024
    t = bench.cpu_prefill_sample(cfg, 40, seed=0)
    assert 0 < t < 60
    gemm, attn = bench.prefill_flops(cfg, [3, 2], world=1)
    H, hd, nq, nkv, inter = 2048, 64, 32, 4, 5632
    params = H * (nq + 2 * nkv) * hd + nq * hd * H + 3 * H * inter
    assert gemm == 2.0 * 5 * params * 2
    assert attn == 4.0 * (6 + 3) * hd * nq * 2  # keys: 1+2+3 and 1+2


def test_reference_arm_prefill_workload_prints_one_json_line():
    env = dict(os.environ, RANK="0")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                          "prefill", "--steps", "1", "--warmup", "0", "--prompts", "2", "--prompt-len", "64"],
                         capture_output=True, text=True, timeout=600, env=env)
    assert out.returncode == 0, out.stderr
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == "prefill tokens/s" and d["value"] > 0


def test_cpu_job_estimate_small_shape():
    import bench
    from pythonintern_b200 import workloads
    cfg = workloads.tinyllama_config(num_layers=2)
    cfg.vocab_size = 1024
    t, desc = bench.cpu_job_estimate(cfg, [20, 36], 2, 64, 3, seed=0)
    assert 0 < t < 120 and "2 prefills" in desc and "3 decode steps" in desc
