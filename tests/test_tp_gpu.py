"""Tensor parallelism over NVLink peer memory (GPU).

* The reference's in-memory all-reduce tests (tests/test_tensor_parallel.py:61-118,
  tests/test_grpc_collectives.py:11-43) with one thread per GPU.
* The vocab-parallel greedy token exchange against torch.argmax over the full row.
* The Tiny LLaMA workload at TP=2 with one process per GPU: greedy tokens identical to
  the reference's TP=2 run.
* A Llama-3-8B-shape bf16 layer at TP=2 against the oracle.
* bench.py's parity leg at TP = 1, 2, 4 and 8 (an 8B-shape layer against the oracle
  fixture, greedy tokens, and at TP <= 2 the Tiny LLaMA tokens of the reference).
* The decode-step sharded all-reduce and the module-level all-reduce at 4 and 8 ranks.
* The timeout path on ONE GPU: rank 1 joins but never enters the all-reduce; rank 0's
  bounded wait runs out and surfaces as TimeoutError (no GPU fault, only rank 0 waits).
Multi-GPU cases skip when fewer GPUs are visible.
"""

import math
import os
import threading

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")
NGPU = torch.cuda.device_count()


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


# ------------------------------------------------------------------ in-process, one thread per GPU
@pytest.mark.skipif(NGPU < 2, reason="needs 2 GPUs")
def test_row_parallel_linear_with_in_memory_comm():
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    from pythonintern_b200.tensor_parallel.layers import RowParallelLinear
    torch.manual_seed(0)
    full = torch.nn.Linear(32, 16, bias=False)
    x = torch.randn(2, 4, 32)
    expected = full(x)
    comms = [DistributedCommunicator(rank=r, world_size=2, device=f"cuda:{r}") for r in range(2)]
    comms[0].register_in_memory_peer(1, comms[1])
    comms[1].register_in_memory_peer(0, comms[0])
    rows = []
    for r in range(2):
        with torch.cuda.device(r):
            m = RowParallelLinear(32, 16, bias=False, rank=r, world_size=2, communicator=comms[r], device=f"cuda:{r}")
            with torch.no_grad():
                m.weight.copy_(full.weight.t()[r * 16:(r + 1) * 16])
            rows.append(m)
    res = [None, None]

    def run(r):
        with torch.cuda.device(r):
            res[r] = rows[r](x[:, :, r * 16:(r + 1) * 16].to(f"cuda:{r}"), step_tag="test_row_parallel").cpu()
    th = [threading.Thread(target=run, args=(r,)) for r in range(2)]
    [t.start() for t in th]
    [t.join() for t in th]
    for r in range(2):
        assert torch.allclose(expected, res[r], atol=1e-5)
    assert torch.equal(res[0], res[1])  # fixed rank-order sum: bit-identical ranks
    for c in comms:
        c.cleanup()


@pytest.mark.skipif(NGPU < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("T", [600, 12000])
def test_sharded_allreduce_rmsnorm_more_rows_than_ctas(T):
    """Prefill-sized calls: 600 rows give each of 2 ranks 300 rows (one CTA per row, more
    rows than the decode grid's 128 CTAs); 12000 rows give 6000, more than can be resident,
    so every CTA reduces several rows.  Against torch float32 on the same inputs."""
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    from pythonintern_b200.tensor_parallel.layers import RowParallelLinear
    K, H, eps = 256, 512, 1e-5
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(T, K, generator=gen).to(torch.bfloat16)
    w = (torch.randn(K, H, generator=gen) * 0.05).to(torch.bfloat16)
    resid = torch.randn(T, H, generator=gen)
    nw = torch.rand(H, generator=gen) + 0.5
    hs = resid + x.float() @ w.float()
    want = hs * torch.rsqrt(hs.pow(2).mean(-1, keepdim=True) + eps) * nw
    comms = [DistributedCommunicator(rank=r, world_size=2, device=f"cuda:{r}") for r in range(2)]
    comms[0].register_in_memory_peer(1, comms[1])
    comms[1].register_in_memory_peer(0, comms[0])
    out = [None, None]
    hout = [None, None]

    def run(r):
        dev = f"cuda:{r}"
        with torch.cuda.device(r):
            m = RowParallelLinear(K, H, bias=False, rank=r, world_size=2, communicator=comms[r],
                                  dtype=torch.bfloat16, device=dev)
            with torch.no_grad():
                m.weight.copy_(w[r * K // 2:(r + 1) * K // 2])
            r0, r1, R = comms[r].row_slice(T)
            h = torch.zeros(R, H, device=dev)
            h[: r1 - r0] = resid[r0:r1].to(dev)
            comms[r].row_parallel_linear(x[:, r * K // 2:(r + 1) * K // 2].contiguous().to(dev), m.packed_weight())
            y = comms[r].allreduce_rmsnorm_sharded(T, H, torch.bfloat16, h, nw.to(dev), eps)
            torch.cuda.synchronize()
            out[r] = y.float().cpu()
            hout[r] = h[: r1 - r0].cpu()
    th = [threading.Thread(target=run, args=(r,)) for r in range(2)]
    [t.start() for t in th]
    [t.join() for t in th]
    for r in range(2):
        assert float((out[r] - want).norm() / want.norm()) < 2e-2
    assert torch.equal(out[0], out[1])  # every rank gets the same all-gathered rows
    got_h = torch.cat(hout)
    assert float((got_h - hs).norm() / hs.norm()) < 1e-2
    for c in comms:
        c.cleanup()


@pytest.mark.parametrize("world", [4, 8])
def test_all_reduce_4_and_8_ranks(world):
    if NGPU < world:
        pytest.skip(f"needs {world} GPUs")
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    comms = [DistributedCommunicator(rank=r, world_size=world, device=f"cuda:{r}") for r in range(world)]
    for i in range(world):
        for j in range(world):
            if i != j:
                comms[i].register_in_memory_peer(j, comms[j])
    res = [None] * world

    def run(r):
        with torch.cuda.device(r):
            t = torch.full((2, 8), float(r + 1), device=f"cuda:{r}")
            res[r] = comms[r].all_reduce_sum(t, step_tag="step_test_collectives").cpu()
    th = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    [t.start() for t in th]
    [t.join() for t in th]
    for r in range(world):
        assert torch.equal(res[r], torch.full((2, 8), float(world * (world + 1) // 2)))
    for c in comms:
        c.cleanup()


@pytest.mark.parametrize("world", [4, 8])
def test_sharded_allreduce_rmsnorm_decode_rows_4_and_8_ranks(world):
    """The decode-step exchange at 4 and 8 ranks: 128 rows of hidden 4096 (the bench's batch),
    every rank pushing its partial rows, three calls in a row (the receive slots rotate),
    against torch float32 on the same inputs; every rank gets identical normalised rows."""
    if NGPU < world:
        pytest.skip(f"needs {world} GPUs")
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    T, K, H, eps = 128, 64 * world, 4096, 1e-5
    gen = torch.Generator().manual_seed(11)
    comms = [DistributedCommunicator(rank=r, world_size=world, device=f"cuda:{r}") for r in range(world)]
    for i in range(world):
        for j in range(world):
            if i != j:
                comms[i].register_in_memory_peer(j, comms[j])
    for call in range(3):
        x = torch.randn(T, K, generator=gen).to(torch.bfloat16)
        w = (torch.randn(K, H, generator=gen) * 0.05).to(torch.bfloat16)
        resid = torch.randn(T, H, generator=gen)
        nw = torch.rand(H, generator=gen) + 0.5
        hs = resid + x.float() @ w.float()
        want = hs * torch.rsqrt(hs.pow(2).mean(-1, keepdim=True) + eps) * nw
        out = [None] * world
        kk = K // world

        def run(r):
            dev = f"cuda:{r}"
            with torch.cuda.device(r):
                wr = w[r * kk:(r + 1) * kk].t().contiguous().to(dev)  # packed [out, in] rows
                r0, r1, R = comms[r].row_slice(T)
                h = torch.zeros(R, H, device=dev)
                h[: r1 - r0] = resid[r0:r1].to(dev)
                comms[r].row_parallel_linear(x[:, r * kk:(r + 1) * kk].contiguous().to(dev), wr)
                y = comms[r].allreduce_rmsnorm_sharded(T, H, torch.bfloat16, h, nw.to(dev), eps)
                torch.cuda.synchronize()
                out[r] = y.float().cpu()
        th = [threading.Thread(target=run, args=(r,)) for r in range(world)]
        [t.start() for t in th]
        [t.join() for t in th]
        for r in range(world):
            assert float((out[r] - want).norm() / want.norm()) < 2e-2, (call, r)
            assert torch.equal(out[r], out[0])
    for c in comms:
        c.cleanup()


@pytest.mark.skipif(NGPU < 2, reason="needs 2 GPUs")
def test_vocab_parallel_argmax_matches_full_argmax():
    """Each rank holds one vocab slice of the logits; the exchanged greedy token equals
    torch.argmax over the full row, ties across the slice boundary and NaN included,
    on several calls in a row (the exchange slots rotate)."""
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    comms = [DistributedCommunicator(rank=r, world_size=2, device=f"cuda:{r}") for r in range(2)]
    comms[0].register_in_memory_peer(1, comms[1])
    comms[1].register_in_memory_peer(0, comms[0])
    V, rows = 1001, 37
    half = (V + 1) // 2
    gen = torch.Generator().manual_seed(3)
    for call in range(4):
        full = torch.randn(rows, V, generator=gen)
        full[0, 10] = full[0, half + 5] = 50.0       # tie across the boundary: the smaller index wins
        full[1, half + 7] = 60.0                       # maximum in the second slice
        full[2, 3] = full[2, 4] = 70.0                 # tie inside the first slice
        full[3, half + 1] = float("nan")               # NaN wins, like torch.argmax
        expected = torch.argmax(full, dim=1)
        res = [None, None]

        def run(r):
            with torch.cuda.device(r):
                v0, v1 = (0, half) if r == 0 else (half, V)
                sl = full[:, v0:v1].contiguous().to(f"cuda:{r}")
                res[r] = comms[r].argmax_allgather(sl, v0).cpu()
        th = [threading.Thread(target=run, args=(r,)) for r in range(2)]
        [t.start() for t in th]
        [t.join() for t in th]
        for r in range(2):
            assert torch.equal(res[r], expected), (call, r)
    for c in comms:
        c.cleanup()


# ------------------------------------------------------------------ one process per GPU
def _tp_tiny_worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from datetime import timedelta
    from pythonintern_b200 import workloads
    from pythonintern_b200.config import KVCacheConfig, ShardConfig
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    from pythonintern_b200.tensor_parallel.sharding import WeightSharder
    from pythonintern_b200.worker.execution_engine import WorkerExecutionEngine
    from pythonintern_b200.worker.messages import SequenceSlot, StepRequest
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    cfg = workloads.tiny_config()
    comm = DistributedCommunicator(rank, world, device=dev).connect()
    eng = WorkerExecutionEngine(cfg, ShardConfig(rank, world), KVCacheConfig(16, 64, str(dev)), comm, dev)
    full = workloads.reference_init_state_dict(cfg, 0)
    eng.model.load_state_dict(WeightSharder(cfg, world).shard_full_model_state_dict(full, rank))
    prompts = workloads.tiny_prompts()
    ids = [f"req_{i}" for i in range(8)]
    for sid, p in zip(ids, prompts):
        eng.kv_manager.allocate_blocks_for_sequence(sid, len(p))
    lens = {sid: len(p) for sid, p in zip(ids, prompts)}
    cur, toks_all = {}, []
    for step in range(32):
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
    np.save(os.path.join(out_dir, f"tokens_rank{rank}.npy"), np.asarray(toks_all))
    dist.barrier()
    comm.cleanup()
    dist.destroy_process_group()


@pytest.mark.skipif(NGPU < 2, reason="needs 2 GPUs")
def test_tiny_workload_tp2_processes(tmp_path):
    gold = np.load(os.path.join(GOLD, "tiny_e2e_tp2.npz"))
    mp.start_processes(_tp_tiny_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    t0 = np.load(tmp_path / "tokens_rank0.npy")
    t1 = np.load(tmp_path / "tokens_rank1.npy")
    assert np.array_equal(t0, t1)
    assert np.array_equal(t0, gold["tokens"])


def _tp_layer_worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from datetime import timedelta
    from pythonintern_b200 import workloads
    from pythonintern_b200.model.kv_cache import PhysicalKVCachePool
    from pythonintern_b200.model.llama import DistributedLLaMAModel
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    from pythonintern_b200.tensor_parallel.sharding import WeightSharder
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    cfg = workloads.llama3_8b_config(num_layers=1, max_seq_len=512)
    cfg.vocab_size = 4096
    sd = workloads.synthetic_state_dict(cfg, seed=21)
    comm = DistributedCommunicator(rank, world, device=dev).connect()
    model = DistributedLLaMAModel(cfg, rank, world, comm, device=dev)
    model.load_state_dict(WeightSharder(cfg, world).shard_full_model_state_dict(sd, rank))
    pool = PhysicalKVCachePool(16, 16, cfg.num_kv_heads // world, cfg.head_dim, 1, dev, "bfloat16")
    toks = torch.randint(0, cfg.vocab_size, (1, 40), generator=torch.Generator().manual_seed(5))
    tr = []
    logits = model(toks.to(dev), torch.arange(40)[None], pool, [[3, 9, 1]], True, 0, trace=tr)
    r0, h_slice = tr[0]
    np.save(os.path.join(out_dir, f"h_rank{rank}.npy"), h_slice.cpu().numpy())
    np.save(os.path.join(out_dir, f"r0_rank{rank}.npy"), np.asarray([r0]))
    np.save(os.path.join(out_dir, f"logits_rank{rank}.npy"), logits.cpu().numpy())
    dist.barrier()
    comm.cleanup()
    dist.destroy_process_group()


@pytest.mark.skipif(NGPU < 2, reason="needs 2 GPUs")
def test_llama3_8b_shape_layer_tp2_matches_oracle(tmp_path):
    import oracle
    from pythonintern_b200 import workloads
    mp.start_processes(_tp_layer_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    # each rank holds the residual of its own rows: rows [0, 20) and [20, 40)
    assert int(np.load(tmp_path / "r0_rank0.npy")[0]) == 0 and int(np.load(tmp_path / "r0_rank1.npy")[0]) == 20
    h0 = np.concatenate([np.load(tmp_path / "h_rank0.npy"), np.load(tmp_path / "h_rank1.npy")])
    assert np.array_equal(np.load(tmp_path / "logits_rank0.npy"), np.load(tmp_path / "logits_rank1.npy"))
    cfg = workloads.llama3_8b_config(num_layers=1, max_seq_len=512)
    cfg.vocab_size = 4096
    sd = {k: v.float().numpy() for k, v in workloads.synthetic_state_dict(cfg, seed=21).items()}
    ocfg = oracle.OracleConfig(cfg.vocab_size, cfg.hidden_dim, 1, cfg.num_heads, cfg.num_kv_heads,
                               cfg.intermediate_dim, cfg.max_seq_len, cfg.rms_norm_eps)
    om = oracle.OracleModel(ocfg, [oracle.shard_state_dict(sd, r, 2) for r in range(2)],
                            [oracle.KVPool(1, 16, 16, cfg.num_kv_heads // 2, cfg.head_dim) for _ in range(2)])
    toks = torch.randint(0, cfg.vocab_size, (1, 40), generator=torch.Generator().manual_seed(5))
    otr = []
    om.forward(toks.numpy(), np.arange(40)[None], [[3, 9, 1]], True, trace=otr)
    err = np.linalg.norm(h0 - otr[0][0]) / np.linalg.norm(otr[0][0])
    assert err < 2e-2


# ------------------------------------------------------------------ bench.py's parity leg at TP = 1, 2, 4, 8
def _parity_worker(rank, world, port, out_dir):
    import json
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from datetime import timedelta
    import bench
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=dev)
    comm = DistributedCommunicator(rank, world, device=dev, max_bytes=64 << 20).connect()
    res = bench.tp_parity(comm, rank, world, dev)
    with open(os.path.join(out_dir, f"parity_rank{rank}.json"), "w") as f:
        json.dump(res, f)
    dist.barrier()
    comm.cleanup()
    dist.destroy_process_group()


def test_parity_leg_tp1():
    """The 8B-shape layer against the oracle fixture and the Tiny LLaMA tokens against the
    reference's golden, at TP=1 (bench.py runs this before timing)."""
    import sys
    sys.path.insert(0, ROOT)
    import bench
    res = bench.tp_parity(None, 0, 1, torch.device("cuda", 0))
    assert res["pass"], res
    assert res["layer_rel_err"] < 2e-2 and res["tokens_checked"] >= 4 and res["tiny_tokens_match"]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_parity_leg_multi_gpu(world, tmp_path):
    """The same check at TP = 2, 4 and 8, one process per GPU (NCCL for the bench's bookkeeping,
    the row-parallel exchange over NVLink peer memory)."""
    import json
    if NGPU < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_parity_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    res = [json.loads((tmp_path / f"parity_rank{r}.json").read_text()) for r in range(world)]
    for r in res:
        assert r == res[0]
    assert res[0]["pass"], res[0]
    assert res[0]["layer_rel_err"] < 2e-2 and res[0]["tokens_checked"] >= 4 and res[0]["ranks_agree"]
    if world == 2:
        assert res[0]["tiny_tokens_match"] is True


# ------------------------------------------------------------------ timeout on one GPU
def _timeout_worker(rank, world, port, out_dir):
    import sys
    import time
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from datetime import timedelta
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    comm = DistributedCommunicator(rank, world, device="cuda:0").connect()
    if rank == 0:
        outcome = "no error"
        t0 = time.time()
        try:
            comm.all_reduce_sum(torch.ones(64, device="cuda:0"), step_tag="lonely", timeout_sec=1.0)
        except TimeoutError as e:
            outcome = "TimeoutError: " + str(e)
        with open(os.path.join(out_dir, "outcome.txt"), "w") as f:
            f.write(f"{outcome}\n{time.time() - t0:.3f}\n")
    # rank 1 never enters the all-reduce; it stays alive (its buffers mapped) until rank 0 is done
    dist.barrier()
    comm.cleanup()
    dist.destroy_process_group()


def test_allreduce_timeout_surfaces_as_timeout_error(tmp_path):
    mp.start_processes(_timeout_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    outcome, secs = (tmp_path / "outcome.txt").read_text().splitlines()
    assert outcome.startswith("TimeoutError"), outcome
    assert "lonely" in outcome
    assert 0.9 < float(secs) < 30.0
