"""Host side of the NVLink communicator on CPU: the IPC-handle exchange that wires the
ranks together, run as world_size-2 gloo process groups (no GPU)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    from datetime import timedelta
    from pythonintern_b200.tensor_parallel.comm import exchange_handles, exchange_handles_store
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    mine = bytes([rank]) * 64
    got = exchange_handles(mine, world)
    assert got == [bytes([r]) * 64 for r in range(world)]
    store = dist.distributed_c10d._get_default_store()
    got2 = exchange_handles_store(store, "test_prefix", rank, world, bytes([7 + rank]) * 64)
    assert got2 == [bytes([7 + r]) * 64 for r in range(world)]
    with open(os.path.join(out_dir, f"ok{rank}"), "w") as f:
        f.write("ok")
    dist.barrier()
    dist.destroy_process_group()


def test_handle_exchange_two_ranks(tmp_path):
    mp.start_processes(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, start_method="spawn")
    assert (tmp_path / "ok0").exists() and (tmp_path / "ok1").exists()


def test_world_size_one_all_reduce_is_identity():
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    c = DistributedCommunicator(0, 1)
    t = torch.ones(3)
    assert c.all_reduce_sum(t, "x") is t  # comm.py:79-80


def test_uncommunicated_rank_refuses():
    from pythonintern_b200.tensor_parallel.comm import DistributedCommunicator
    c = DistributedCommunicator(0, 2)
    with pytest.raises(RuntimeError):
        c._require_open()
