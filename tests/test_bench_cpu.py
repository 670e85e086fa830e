"""The CPU legs of bench.py (the reference-algorithm arm) run without a GPU."""

import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_cpu_sample_small_shape():
    import bench
    from pythonintern_b200 import workloads
    cfg = workloads.tinyllama_config(num_layers=2)
    cfg.vocab_size = 1024
    t = bench.cpu_sample(cfg, batch=2, ctx=64, seed=0)
    assert 0 < t < 60


def test_reference_arm_prints_one_json_line():
    env = dict(os.environ, RANK="0")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--cpu-sample-batch", "1", "--ctx", "64"],
                         capture_output=True, text=True, timeout=600, env=env)
    assert out.returncode == 0, out.stderr
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"]["h2d_bytes_per_step"] == 0


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
