"""The CPU restatement of the reference's gRPC tensor-parallel decode (oracle/grpc_tp.py).

It is the timed stand-in for the reference in bench.py's reference arm, so it is
checked here against the numpy oracle (itself pinned to the reference's golden
vectors): the batched decode attention, one rank's decoder layer, the protobuf wire
message and the all-reduce over real gRPC channels on localhost.
"""

import math
import threading

import numpy as np
import torch

import oracle
from oracle import decoder as od
from oracle import grpc_tp


def test_batched_decode_attention_matches_oracle():
    rng = np.random.default_rng(0)
    B, nq, nkv, hd = 3, 8, 2, 16
    kc = rng.standard_normal((1, 12, 16, nkv, hd))
    vc = rng.standard_normal((1, 12, 16, nkv, hd))
    pool = od.KVPool(1, 12, 16, nkv, hd, dtype=np.float64)
    pool.k[:], pool.v[:] = kc, vc
    q = rng.standard_normal((B, nq, hd))
    k = rng.standard_normal((B, nkv, hd))
    v = rng.standard_normal((B, nkv, hd))
    pos = np.array([5, 33, 20])
    tables = [[0, 1], [2, 3, 4], [5, 6]]
    want = od.decode_attention(q, k, v, pos, pool, 0, tables, 0.25, compat_pad=True)
    kt, vt = torch.from_numpy(kc.copy()), torch.from_numpy(vc.copy())
    got = grpc_tp.decode_attention_batched(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v),
                                           torch.from_numpy(pos), kt, vt, 0, tables, 0.25)
    assert np.abs(got.numpy() - want).max() < 1e-12
    assert np.array_equal(kt.numpy(), pool.k) and np.array_equal(vt.numpy(), pool.v)


def test_rank_layer_matches_oracle_block():
    """World 1: RankLayer.decode (torch float32) against oracle.OracleModel.block (float64)."""
    H, nq, nkv, inter, B, ctx = 64, 4, 2, 96, 3, 40
    lay = grpc_tp.RankLayer(H, nq, nkv, inter, 0, 1, B, ctx, seed=3)
    w = {k: v.numpy().astype(np.float64) for k, v in lay.w.items()}
    shard = {"layers.0.input_layernorm.weight": w["n1"], "layers.0.post_attention_layernorm.weight": w["n2"],
             "layers.0.self_attn.q_proj.weight": w["q"], "layers.0.self_attn.k_proj.weight": w["k"],
             "layers.0.self_attn.v_proj.weight": w["v"], "layers.0.self_attn.out_proj.weight": w["o"],
             "layers.0.mlp.gate_proj.weight": w["g"], "layers.0.mlp.up_proj.weight": w["u"],
             "layers.0.mlp.down_proj.weight": w["d"]}
    pool = od.KVPool(1, lay.k_cache.shape[1], 16, nkv, H // nq, dtype=np.float64)
    pool.k[:], pool.v[:] = lay.k_cache.numpy(), lay.v_cache.numpy()
    cfg = oracle.OracleConfig(16, H, 1, nq, nkv, inter, ctx + 64, 1e-5)
    om = oracle.OracleModel(cfg, [shard], [pool])
    h = torch.randn(B, 1, H, generator=torch.Generator().manual_seed(1))
    pos = torch.tensor([[ctx - 1], [ctx - 9], [ctx - 30]])
    comm = grpc_tp.GrpcAllReduce(0, 1)
    got = lay.decode(h, pos, 0, comm).numpy()
    want = om.block(0, h.numpy().astype(np.float64), pos.numpy(), lay.tables, False)
    assert np.abs(got - want).max() / np.abs(want).max() < 1e-5


def test_wire_message_round_trip():
    Payload, Response = grpc_tp.wire_classes()
    t = torch.randn(3, 5)
    raw, shape, dt = grpc_tp.serialize_tensor(t)
    msg = Payload(step_tag="step_1_l0_attn", sender_rank=1, shape=list(shape), dtype=dt, raw_tensor_data=raw)
    back = Payload.FromString(msg.SerializeToString())
    assert back.step_tag == "step_1_l0_attn" and back.sender_rank == 1 and list(back.shape) == [3, 5]
    got = grpc_tp.deserialize_tensor(back.raw_tensor_data, back.shape, back.dtype)
    assert torch.equal(got, t)
    assert Response.FromString(Response(success=True).SerializeToString()).success


def test_grpc_all_reduce_three_ranks_localhost():
    """Three communicators in one process, each with its own gRPC server on localhost."""
    world = 3
    ports = grpc_tp.free_ports(world)
    comms = [grpc_tp.GrpcAllReduce(r, world) for r in range(world)]
    for r, c in enumerate(comms):
        c.serve(ports[r])
    for c in comms:
        c.connect([f"127.0.0.1:{p}" for p in ports])
    res = [None] * world

    def run(r):
        res[r] = comms[r].all_reduce_sum(torch.full((2, 4), float(r + 1)), "step_0_l0_attn", timeout_sec=30)
    th = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    [t.start() for t in th]
    [t.join() for t in th]
    for r in range(world):
        assert torch.equal(res[r], torch.full((2, 4), 6.0))
    for c in comms:
        c.cleanup()


def test_grpc_all_reduce_timeout_names_the_tag():
    ports = grpc_tp.free_ports(2)
    c0, c1 = grpc_tp.GrpcAllReduce(0, 2), grpc_tp.GrpcAllReduce(1, 2)
    c0.serve(ports[0])
    c1.serve(ports[1])
    c0.connect([f"127.0.0.1:{p}" for p in ports])
    try:
        c0.all_reduce_sum(torch.ones(4), "lonely", timeout_sec=0.5)
        raise AssertionError("expected TimeoutError")
    except TimeoutError as e:
        assert "lonely" in str(e)
    finally:
        c0.cleanup()
        c1.cleanup()
