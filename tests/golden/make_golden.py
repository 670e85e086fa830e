"""Generate the golden vectors that pin the oracle to the reference engine.

Runs the UNMODIFIED reference (kmadasamy212-tech/pythonintern, a read-only checkout
whose path is the first argument or ``$PYTHONINTERN_REFERENCE``) on CPU and writes
small fixtures next to this script:

* ``tiny_weights_fingerprint.json`` - sha256 of every tensor of the seed-0 Tiny
  LLaMA state dict the reference builds (so the seed-0 weights can be regenerated
  without the reference, see ``pythonintern_b200.workloads.reference_init_state_dict``).
* ``tiny_e2e_tp1.npz`` / ``tiny_e2e_tp2.npz`` - the Tiny LLaMA greedy workload
  (8 prompts, 32 greedy tokens) driven through ``WorkerExecutionEngine.execute_step``
  with a correct block allocator: tokens, top_logits, block tables and per-layer
  activations of the first prefill and the first decode step.
* ``units.npz`` - seeded inputs and outputs of the individual hot-path functions
  (RoPE tables and apply, RMSNorm, column/row-parallel linears with the in-memory
  all-reduce, paged KV store/read, attention prefill/decode, SwiGLU MLP, block).

The reference's generated protobuf stubs were produced by a newer protoc than the
installed runtime, so the two version checks are disabled before import.

Usage:  python tests/golden/make_golden.py <reference checkout>   (CPU only)
"""

import hashlib
import json
import math
import os
import sys
import threading

import numpy as np
import torch

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PYTHONINTERN_REFERENCE", "")
if not REF or not os.path.isdir(os.path.join(REF, "engine")):
    sys.exit("usage: make_golden.py <path to a kmadasamy212-tech/pythonintern checkout> "
             "(or set PYTHONINTERN_REFERENCE)")
REF = os.path.abspath(REF)
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.dont_write_bytecode = True


def import_reference():
    import google.protobuf.runtime_version as rv
    rv.ValidateProtobufRuntimeVersion = lambda *a, **k: None
    import grpc._utilities as gu
    gu.first_version_is_lower = lambda a, b: False
    if REF not in sys.path:
        sys.path.insert(0, REF)
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)


import_reference()
from engine.config import ModelConfig as RModelConfig, ShardConfig, KVCacheConfig  # noqa: E402
from engine.model.attention import DistributedAttention, RotaryEmbedding  # noqa: E402
from engine.model.kv_cache import BlockTable, PhysicalKVCachePool  # noqa: E402
from engine.model.llama import DistributedLLaMAModel, DistributedTransformerBlock  # noqa: E402
from engine.model.mlp import DistributedMLP  # noqa: E402
from engine.tensor_parallel.comm import DistributedCommunicator  # noqa: E402
from engine.tensor_parallel.layers import ColumnParallelLinear, RowParallelLinear, RMSNorm  # noqa: E402
from engine.tensor_parallel.sharding import WeightSharder  # noqa: E402
from engine.worker.execution_engine import WorkerExecutionEngine  # noqa: E402
import proto_gen.distributed_inference_pb2 as pb2  # noqa: E402

from pythonintern_b200 import workloads  # noqa: E402

torch.set_num_threads(8)


def tiny_ref_config():
    c = workloads.tiny_config()
    return RModelConfig(vocab_size=c.vocab_size, hidden_dim=c.hidden_dim, num_layers=c.num_layers,
                        num_heads=c.num_heads, num_kv_heads=c.num_kv_heads,
                        intermediate_dim=c.intermediate_dim, max_seq_len=c.max_seq_len,
                        rms_norm_eps=c.rms_norm_eps)


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().numpy().tobytes()).hexdigest()


def make_comms(ws):
    comms = [DistributedCommunicator(rank=r, world_size=ws) for r in range(ws)]
    for i in range(ws):
        for j in range(ws):
            if i != j:
                comms[i].register_in_memory_peer(j, comms[j])
    return comms


def run_ranks(fns):
    res = [None] * len(fns)
    errs = []

    def wrap(i):
        try:
            res[i] = fns[i]()
        except Exception as e:  # pragma: no cover - surfaced below
            errs.append(e)
    th = [threading.Thread(target=wrap, args=(i,)) for i in range(len(fns))]
    for t in th:
        t.start()
    for t in th:
        t.join()
    if errs:
        raise errs[0]
    return res


# ------------------------------------------------------------------------------------------
# Tiny LLaMA end to end
# ------------------------------------------------------------------------------------------

def tiny_e2e(ws: int, full_sd, num_tokens=32, num_blocks=64):
    cfg = tiny_ref_config()
    comms = make_comms(ws)
    engines = []
    for r in range(ws):
        eng = WorkerExecutionEngine(cfg, ShardConfig(rank=r, world_size=ws), KVCacheConfig(16, num_blocks),
                                    comms[r], device="cpu")
        shard = WeightSharder(cfg, ws).shard_full_model_state_dict(full_sd, r)
        eng.model.load_state_dict(shard)
        eng.model.eval()
        engines.append(eng)
    traces = {"prefill": [], "decode": []}
    mode = {"cur": None}
    hooks = []
    for i, layer in enumerate(engines[0].model.layers):
        def hook(mod, inp, out, i=i):
            if mode["cur"] is not None:
                traces[mode["cur"]].append(out.detach().clone())
        hooks.append(layer.register_forward_hook(hook))

    orig_forward = engines[0].model.forward
    calls = {"n": 0}
    n_prompts = len(workloads.tiny_prompts())

    def counting_forward(*a, **k):
        n = calls["n"]
        calls["n"] += 1
        mode["cur"] = "prefill" if n == 0 else ("decode" if n == n_prompts else None)
        return orig_forward(*a, **k)
    engines[0].model.forward = counting_forward

    prompts = workloads.tiny_prompts()
    ids = [f"req_{i}" for i in range(len(prompts))]
    lens = {}
    for sid, p in zip(ids, prompts):
        for e in engines:
            e.kv_manager.allocate_blocks_for_sequence(sid, len(p))
        lens[sid] = len(p)

    def tables():
        return {sid: list(engines[0].kv_manager.block_tables[sid].physical_block_ids) for sid in ids}

    all_tokens, all_tops = [], []
    cur = {}
    for step in range(num_tokens):
        if step == 0:
            slots = [pb2.SequenceSlotProto(seq_id=sid, is_prefill=True, prompt_token_ids=p,
                                           current_len=len(p), block_table=tables()[sid])
                     for sid, p in zip(ids, prompts)]
        else:
            for sid in ids:
                for e in engines:
                    e.kv_manager.append_token(sid)
                lens[sid] += 1
            tb = tables()
            slots = [pb2.SequenceSlotProto(seq_id=sid, is_prefill=False, current_token_id=cur[sid],
                                           current_len=lens[sid], block_table=tb[sid]) for sid in ids]
        req = pb2.StepRequest(step_id=step, active_sequences=slots)
        resps = run_ranks([lambda e=e: e.execute_step(req) for e in engines])
        for r in resps:
            assert r.success, r.error_message
        toks = [t.token_id for t in resps[0].sampled_tokens]
        tops = [list(t.top_logits) for t in resps[0].sampled_tokens]
        assert [t.seq_id for t in resps[0].sampled_tokens] == ids
        for r in resps[1:]:
            assert [t.token_id for t in r.sampled_tokens] == toks, "ranks disagree"
        cur = dict(zip(ids, toks))
        all_tokens.append(toks)
        all_tops.append(tops)
    for h in hooks:
        h.remove()
    tb = tables()
    max_nb = max(len(v) for v in tb.values())
    tab = np.full((len(ids), max_nb), -1, dtype=np.int32)
    for i, sid in enumerate(ids):
        tab[i, :len(tb[sid])] = tb[sid]
    out = dict(
        tokens=np.asarray(all_tokens, dtype=np.int64),
        top_logits=np.asarray(all_tops, dtype=np.float32),
        block_tables=tab,
        prompt_lens=np.asarray([len(p) for p in prompts], dtype=np.int64),
        prefill_trace=torch.stack([t[0] for t in traces["prefill"]]).numpy(),   # [L, P0, H]
        decode_trace=torch.stack([t[:, 0] for t in traces["decode"]]).numpy(),  # [L, B, H]
    )
    for c in comms:
        c.cleanup()
    return out


# ------------------------------------------------------------------------------------------
# Unit goldens
# ------------------------------------------------------------------------------------------

def unit_goldens():
    g = {}
    torch.manual_seed(1234)
    # RoPE tables (attention.py:35-44) and apply (:46-63)
    for hd in (32, 64, 128):
        rope = RotaryEmbedding(hd, max_seq_len=2048)
        rows = np.r_[0:96, 500, 1023, 1024, 2047]
        g[f"rope{hd}_rows"] = rows
        g[f"rope{hd}_cos"] = rope.cos_cached[rows].numpy()
        g[f"rope{hd}_sin"] = rope.sin_cached[rows].numpy()
    rope = RotaryEmbedding(32, max_seq_len=2048)
    x = torch.randn(2, 5, 4, 32)
    pos = torch.tensor([[0, 1, 2, 3, 4], [100, 37, 2046, 5, 999]])
    g["rope_apply_x"], g["rope_apply_pos"] = x.numpy(), pos.numpy()
    g["rope_apply_y"] = rope.apply_rope(x, pos).numpy()

    # RMSNorm (layers.py:165-184)
    norm = RMSNorm(64, eps=1e-5)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(64) + 0.5)
    x = torch.randn(2, 5, 64) * 3
    g["rms_x"], g["rms_w"], g["rms_y"] = x.numpy(), norm.weight.detach().numpy(), norm(x).detach().numpy()

    # Column-parallel (layers.py:23-86), two ranks, reference test shapes
    full = torch.nn.Linear(32, 64, bias=False)
    x = torch.randn(2, 4, 32)
    cols = []
    for r in range(2):
        m = ColumnParallelLinear(32, 64, bias=False, rank=r, world_size=2)
        with torch.no_grad():
            m.weight.copy_(full.weight.t()[:, r * 32:(r + 1) * 32])
            cols.append(m(x).numpy())
    g["col_x"], g["col_w_full"] = x.numpy(), full.weight.t().detach().contiguous().numpy()
    g["col_y_r0"], g["col_y_r1"] = cols

    # Row-parallel + in-memory all-reduce (layers.py:89-162, comm.py:72-118), two ranks
    full = torch.nn.Linear(32, 16, bias=False)
    x = torch.randn(2, 4, 32)
    comms = make_comms(2)
    mods = [RowParallelLinear(32, 16, bias=False, rank=r, world_size=2, communicator=comms[r]) for r in range(2)]
    with torch.no_grad():
        for r in range(2):
            mods[r].weight.copy_(full.weight.t()[r * 16:(r + 1) * 16])
        ys = run_ranks([lambda r=r: mods[r](x[:, :, r * 16:(r + 1) * 16], step_tag="row") for r in range(2)])
    g["row_x"], g["row_w_full"] = x.numpy(), full.weight.t().detach().contiguous().numpy()
    g["row_y_r0"], g["row_y_r1"] = ys[0].detach().numpy(), ys[1].detach().numpy()

    # 4-rank all-reduce of (r+1)*ones (tests/test_grpc_collectives.py:11-43)
    comms = make_comms(4)
    ys = run_ranks([lambda r=r: comms[r].all_reduce_sum(torch.full((2, 8), float(r + 1)), "ar4") for r in range(4)])
    g["ar4_y"] = np.stack([y.detach().numpy() for y in ys])

    # Block-table slots (kv_cache.py:35-43)
    bt = BlockTable("s", 16)
    for b in (4, 9, 2, 7):
        bt.append_block(b)
    q = np.arange(64)
    g["slot_pos"] = q
    g["slot_out"] = np.asarray([bt.get_physical_slot(int(p)) for p in q], dtype=np.int64)

    # Paged pool roundtrip with a permuted table (kv_cache.py:85-147)
    pool = PhysicalKVCachePool(num_blocks=12, block_size=16, num_local_kv_heads=2, head_dim=32, num_layers=2)
    table = [7, 3, 10, 0]
    kk, vv = torch.randn(50, 2, 32), torch.randn(50, 2, 32)
    for t in range(50):
        pool.store_kv(1, table[t // 16], t % 16, kk[t], vv[t])
    ks, vs = pool.read_kv_sequence(1, table, 41)
    g["pool_k_in"], g["pool_v_in"], g["pool_table"] = kk.numpy(), vv.numpy(), np.asarray(table)
    g["pool_k_out"], g["pool_v_out"] = ks.numpy(), vs.numpy()
    g["pool_k_cache"] = pool.k_cache.numpy()

    # Attention: prefill two prompts (batch 1 each), then one decode step of both
    # (different context lengths => the reference's unmasked zero padding).
    cfg = RModelConfig(vocab_size=64, hidden_dim=128, num_layers=1, num_heads=4, num_kv_heads=2,
                       intermediate_dim=96, max_seq_len=256)
    torch.manual_seed(7)
    attn = DistributedAttention(cfg, layer_idx=0)
    pool = PhysicalKVCachePool(num_blocks=16, block_size=16, num_local_kv_heads=2, head_dim=32, num_layers=1)
    tables = [[5, 2, 11], [9, 0, 14]]
    lens = [21, 6]
    with torch.no_grad():
        for b in range(2):
            xp = torch.randn(1, lens[b], 128)
            yp = attn(xp, torch.arange(lens[b])[None], pool, [tables[b]], True, 0)
            g[f"attn_prefill{b}_x"], g[f"attn_prefill{b}_y"] = xp.numpy(), yp.numpy()
        xd = torch.randn(2, 1, 128)
        posd = torch.tensor([[lens[0]], [lens[1]]])
        yd = attn(xd, posd, pool, tables, False, 1)
    g["attn_decode_x"], g["attn_decode_pos"], g["attn_decode_y"] = xd.numpy(), posd.numpy(), yd.numpy()
    g["attn_tables"], g["attn_lens"] = np.asarray(tables), np.asarray(lens)
    for n in ("q_proj", "k_proj", "v_proj", "out_proj"):
        g[f"attn_{n}"] = getattr(attn, n).weight.detach().numpy()
    g["attn_k_cache"], g["attn_v_cache"] = pool.k_cache.numpy(), pool.v_cache.numpy()

    # SwiGLU MLP (mlp.py:22-86)
    torch.manual_seed(8)
    mlp = DistributedMLP(cfg, layer_idx=0)
    x = torch.randn(3, 2, 128)
    with torch.no_grad():
        g["mlp_x"], g["mlp_y"] = x.numpy(), mlp(x).numpy()
    for n in ("gate_proj", "up_proj", "down_proj"):
        g[f"mlp_{n}"] = getattr(mlp, n).weight.detach().numpy()

    # Transformer block (llama.py:25-76): prefill 5 tokens then one decode token
    torch.manual_seed(9)
    blk = DistributedTransformerBlock(cfg, layer_idx=0)
    with torch.no_grad():
        blk.input_layernorm.weight.copy_(torch.rand(128) + 0.5)
        blk.post_attention_layernorm.weight.copy_(torch.rand(128) + 0.5)
    pool = PhysicalKVCachePool(num_blocks=4, block_size=16, num_local_kv_heads=2, head_dim=32, num_layers=1)
    with torch.no_grad():
        xp = torch.randn(1, 5, 128)
        yp = blk(xp, torch.arange(5)[None], pool, [[3]], True, 0)
        xd = torch.randn(1, 1, 128)
        yd = blk(xd, torch.tensor([[5]]), pool, [[3]], False, 1)
    g["blk_xp"], g["blk_yp"], g["blk_xd"], g["blk_yd"] = xp.numpy(), yp.numpy(), xd.numpy(), yd.numpy()
    for k, v in blk.state_dict().items():
        g["blk." + k] = v.numpy()
    return g


def main():
    cfg = tiny_ref_config()
    torch.manual_seed(0)
    ref_model = DistributedLLaMAModel(cfg)
    ref_sd = {k: v.detach().clone() for k, v in ref_model.state_dict().items()}
    ours = workloads.reference_init_state_dict(workloads.tiny_config(), seed=0)
    assert list(ours.keys()) == list(ref_sd.keys()), "key order differs"
    for k in ref_sd:
        assert torch.equal(ours[k], ref_sd[k]), f"seed-0 replay differs at {k}"
    fp = {k: sha(v) for k, v in ref_sd.items()}
    with open(os.path.join(HERE, "tiny_weights_fingerprint.json"), "w") as f:
        json.dump(fp, f, indent=1, sort_keys=False)

    for ws in (1, 2):
        out = tiny_e2e(ws, ref_sd)
        np.savez_compressed(os.path.join(HERE, f"tiny_e2e_tp{ws}.npz"), **out)
        print(f"tp{ws}: tokens[0]={out['tokens'][0].tolist()} tokens[-1]={out['tokens'][-1].tolist()}")
    np.savez_compressed(os.path.join(HERE, "units.npz"), **unit_goldens())
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
