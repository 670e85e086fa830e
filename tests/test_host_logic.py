"""Host-side logic that needs no GPU: configuration, block tables and the FIFO allocator,
token metadata, weight sharding, step messages, seeded workloads."""

import dataclasses
import math
import sys

import numpy as np
import pytest
import torch

import oracle
from pythonintern_b200 import config, workloads
from pythonintern_b200.model.kv_cache import BlockTable, KVCacheManager
from pythonintern_b200.model.metadata import build_metadata, pad_tables
from pythonintern_b200.tensor_parallel.sharding import WeightSharder
from pythonintern_b200.worker.messages import SampledToken, StepResponse


def test_config_fields_match_the_reference():
    names = [f.name for f in dataclasses.fields(config.ModelConfig)]
    for n in ("vocab_size", "hidden_dim", "num_layers", "num_heads", "num_kv_heads", "intermediate_dim",
              "max_seq_len", "rms_norm_eps", "rope_theta", "dtype"):
        assert n in names
    c = config.ModelConfig()
    assert (c.vocab_size, c.hidden_dim, c.num_layers, c.num_heads, c.num_kv_heads, c.intermediate_dim) == \
        (32000, 1024, 8, 16, 4, 2816)
    assert c.head_dim == 64 and c.rope_base == 10000.0
    c8 = workloads.llama3_8b_config()
    assert c8.rope_theta == 500000.0 and c8.rope_base == 10000.0  # the reference ignores rope_theta
    c8.honor_rope_theta = True
    assert c8.rope_base == 500000.0
    assert config.KVCacheConfig().block_size == 16


def test_block_table_slots():
    """tests/test_kv_cache.py:11-23."""
    bt = BlockTable("seq_1", block_size=16)
    bt.append_block(4)
    bt.append_block(9)
    assert bt.get_physical_slot(5) == (4, 5)
    assert bt.get_physical_slot(16) == (9, 0)
    assert bt.get_physical_slot(20) == (9, 4)
    with pytest.raises(AssertionError):
        bt.get_physical_slot(32)


def test_kv_manager_matches_oracle_allocator():
    mgr = KVCacheManager(config.KVCacheConfig(block_size=16, num_blocks=40, device="meta"),
                         config.ModelConfig(hidden_dim=64, num_heads=4, num_kv_heads=2, num_layers=2), world_size=1)
    ref = oracle.FifoBlockAllocator(40, 16)
    for i, n in enumerate([30, 1, 16, 17, 64]):
        assert mgr.allocate_blocks_for_sequence(f"s{i}", n).physical_block_ids == ref.allocate(f"s{i}", n)
    for _ in range(20):
        for i in range(5):
            assert mgr.append_token(f"s{i}") == ref.append_token(f"s{i}")
    assert mgr.free_sequence("s2") == len(ref.tables["s2"])
    assert mgr.free_sequence("missing") == 0
    with pytest.raises(MemoryError):
        mgr.allocate_blocks_for_sequence("big", 16 * 100)


def test_decode_metadata():
    md = build_metadata(np.array([[39], [30], [0]]), [[3, 4, 5], [7, 1], [2]], False, "cpu")
    assert md.n_tokens == 3 and not md.is_prefill and md.compat_pad
    assert md.rope_pos.tolist() == [39, 30, 0]
    assert md.store_pos is None and md.table_index is None
    assert md.ctx_lens.tolist() == [40, 31, 1] and md.max_ctx == 40
    assert md.tables.tolist() == [[3, 4, 5], [7, 1, -1], [2, -1, -1]]
    assert md.tables.dtype == torch.int32
    md2 = build_metadata(np.array([[39]]), [[3, 4, 5]], False, "cpu", masked_padding=True)
    assert not md2.compat_pad


def test_prefill_metadata_causal_rows():
    md = build_metadata(np.arange(5)[None] + 100, [[9]], True, "cpu")
    assert md.rope_pos.tolist() == [100, 101, 102, 103, 104]  # rotation uses positions
    assert md.store_pos.tolist() == [0, 1, 2, 3, 4]            # storage uses t (attention.py:170-173)
    assert md.table_index.tolist() == [0] * 5
    assert md.ctx_lens.tolist() == [1, 2, 3, 4, 5] and not md.compat_pad


def test_pad_tables_empty():
    assert pad_tables([[], [1]]).tolist() == [[-1], [1]]


@pytest.mark.parametrize("ws", [1, 2])
def test_weight_sharder_matches_oracle(ws):
    cfg = workloads.tiny_config()
    full = workloads.reference_init_state_dict(cfg, 0)
    ours = WeightSharder(cfg, ws)
    for r in range(ws):
        a = ours.shard_full_model_state_dict(full, r)
        b = oracle.shard_state_dict({k: v.numpy() for k, v in full.items()}, r, ws)
        assert list(a) == list(b)
        for k in a:
            assert np.array_equal(a[k].numpy(), b[k]), k


def test_step_response_to_proto_with_fake_module():
    class Msg:
        def __init__(self, **kw):
            self.__dict__.update(kw)

    class FakePb2:
        StepResponse = Msg
        SampledTokenProto = Msg

    r = StepResponse(3, 1, True, sampled_tokens=[SampledToken("a", 5, [1.0])], step_latency_ms=2.0)
    p = r.to_proto(FakePb2)
    assert p.step_id == 3 and p.sampled_tokens[0].token_id == 5 and p.sampled_tokens[0].seq_id == "a"


def test_synthetic_weights_deterministic():
    cfg = workloads.tinyllama_config(num_layers=1)
    cfg.vocab_size = 128
    a = workloads.synthetic_state_dict(cfg, seed=3)
    b = workloads.synthetic_state_dict(cfg, seed=3)
    assert all(torch.equal(a[k], b[k]) for k in a)
    assert a["layers.0.self_attn.q_proj.weight"].dtype == torch.bfloat16
    assert abs(float(a["layers.0.mlp.up_proj.weight"].float().std()) - 0.02) < 1e-3


def test_package_has_no_cpu_compute_path():
    """The compute modules raise instead of falling back when tensors are on the CPU."""
    from pythonintern_b200 import kernels
    with pytest.raises(Exception):
        kernels.linear(torch.zeros(2, 8), torch.zeros(4, 8))


def test_decode_graph_packs_only_changed_table_rows():
    """The decode graph's host packing reuses the previous step's rows and rewrites a row
    only when its block table changed (grown, shrunk or edited), padding with -1."""
    from types import SimpleNamespace
    from pythonintern_b200.worker.graphs import DecodeGraph, _layout
    B, W = 3, 8
    g = SimpleNamespace(batch=B, width=W, _tab=np.full((B, W), -1, dtype=np.int32), _rows=[None] * B)
    total = _layout(B, W)[-1]
    out = np.zeros(total, dtype=np.uint8)
    o_tab = _layout(B, W)[3]

    def tabs():
        return out[o_tab:o_tab + 4 * B * W].view(np.int32).reshape(B, W)
    tables = [[5, 6], [7], [1, 2, 3]]
    DecodeGraph.pack(g, [1, 2, 3], [10, 11, 12], tables, out)
    assert tabs().tolist() == [[5, 6] + [-1] * 6, [7] + [-1] * 7, [1, 2, 3] + [-1] * 5]
    tables = [[5, 6, 9], [4], np.array([1, 2, 3])]  # grown, edited, unchanged (as an array)
    DecodeGraph.pack(g, [1, 2, 3], [10, 11, 12], tables, out)
    assert tabs().tolist() == [[5, 6, 9] + [-1] * 5, [4] + [-1] * 7, [1, 2, 3] + [-1] * 5]
    DecodeGraph.pack(g, [1, 2, 3], [10, 11, 12], [[5], [4], [1, 2, 3]], out)  # shrunk
    assert tabs()[0].tolist() == [5] + [-1] * 7
    with pytest.raises(ValueError):
        DecodeGraph.pack(g, [1, 2, 3], [10, 11, 12], [[0] * (W + 1), [4], [1]], out)


def test_vocab_slices_cover_the_vocabulary_once():
    """Each rank's lm_head rows for the vocab-parallel greedy step: contiguous, disjoint,
    covering [0, V) in rank order (so rank order is vocabulary order)."""
    from types import SimpleNamespace
    from pythonintern_b200.model.llama import DistributedLLaMAModel
    for V in (1024, 32000, 128256, 1001):
        for t in (1, 2, 4, 8):
            spans = [DistributedLLaMAModel.vocab_slice(SimpleNamespace(config=SimpleNamespace(vocab_size=V),
                                                                       world_size=t, rank=r)) for r in range(t)]
            assert spans[0][0] == 0 and spans[-1][1] == V
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(e > s for s, e in spans)


def test_prefill_layout_positions_and_sequence_bounds():
    from pythonintern_b200.model.metadata import prefill_layout
    pos, tidx, ctx, seq_start, last, c0 = prefill_layout([3, 1, 2])
    assert pos.tolist() == [0, 1, 2, 0, 0, 1]  # arange(P) per prompt (execution_engine.py:88-93)
    assert tidx.tolist() == [0, 0, 0, 1, 2, 2]
    assert ctx.tolist() == [1, 2, 3, 1, 1, 2]
    assert seq_start.tolist() == [0, 3, 4, 6] and seq_start.dtype == np.int32
    assert last.tolist() == [2, 3, 5] and c0 is None
    pos, _, ctx, _, _, c0 = prefill_layout([2, 2], ctx0=[0, 16])
    assert pos.tolist() == [0, 1, 16, 17] and ctx.tolist() == [1, 2, 17, 18] and c0.tolist() == [0, 16]
    for bad in ([], [2, 0], [-1]):
        with pytest.raises(ValueError):
            prefill_layout(bad)
    with pytest.raises(ValueError):
        prefill_layout([2], ctx0=[-1])


def test_group_prefills_respects_the_token_cap():
    from pythonintern_b200.worker.execution_engine import group_prefills
    assert group_prefills([60, 30, 20, 150, 5], 100) == [[0, 1], [2], [3], [4]]
    assert group_prefills([10, 10, 10], 100) == [[0, 1, 2]]
    assert group_prefills([10, 10, 10], 100, batch=False) == [[0], [1], [2]]
    assert group_prefills([], 100) == []


# ------------------------------------------------------------------ coordinator block allocator
class _Seq:
    def __init__(self, seq_id, prompt_len):
        self.seq_id = seq_id
        self.prompt_token_ids = list(range(prompt_len))
        self.output_token_ids = []

    @property
    def total_length(self):
        return len(self.prompt_token_ids) + len(self.output_token_ids)


def _drive(mm, prompt_len, steps):
    """The reference batcher's order: allocate the prompt, sample a token, then per decode step
    append_token_slot before the worker writes position total_length - 1, then sample."""
    s = _Seq("s", prompt_len)
    mm.allocate_prefill(s)
    s.output_token_ids.append(0)
    short = []
    for _ in range(steps):
        mm.append_token_slot(s)
        pos = s.total_length - 1
        short.append(pos // mm.block_size >= len(mm.get_block_table("s")))
        s.output_token_ids.append(0)
    return short


def test_cluster_memory_manager_reproduces_the_off_by_one_by_default():
    """Prompts of 16 and 32 tokens reach their first decode with a table one block short
    (engine/scheduler/memory_manager.py:54-74); other lengths do not."""
    from pythonintern_b200.config import KVCacheConfig
    from pythonintern_b200.scheduler import ClusterMemoryManager
    for P in (16, 32):
        assert _drive(ClusterMemoryManager(KVCacheConfig(16, 64, "cuda")), P, 3)[0] is True
    assert not any(_drive(ClusterMemoryManager(KVCacheConfig(16, 64, "cuda")), 17, 40))


def test_cluster_memory_manager_fixed_allocator_always_covers_the_written_slot():
    from pythonintern_b200.config import KVCacheConfig
    from pythonintern_b200.scheduler import ClusterMemoryManager
    for P in (1, 15, 16, 17, 31, 32, 33, 64):
        mm = ClusterMemoryManager(KVCacheConfig(16, 64, "cuda"), fixed_allocator=True)
        assert not any(_drive(mm, P, 50)), P
        # never more blocks than the tokens need
        assert len(mm.get_block_table("s")) == math.ceil((P + 50) / 16)
    mm = ClusterMemoryManager(KVCacheConfig(16, 64, "cuda"), fixed_allocator=True)
    a, b = _Seq("a", 20), _Seq("b", 5)
    assert mm.allocate_prefill(a) == [0, 1] and mm.allocate_prefill(b) == [2]   # FIFO pop(0)
    assert mm.free_sequence(a) == [0, 1] and mm.free_blocks[-2:] == [0, 1]
