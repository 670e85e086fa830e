"""Varlen causal prefill (``b2_prefill_attention``) and the batched prefill step (GPU).

The reference runs every prompt as its own batch-1 forward with a causal mask over its
in-flight keys (engine/model/attention.py:166-174,211-228; execution_engine.py:85-111).
Here all prompts of a step go through one forward and one attention launch per layer.
Checked against the oracle: per row, the masked single-token attention at that position
(``oracle.decode_attention`` with ``compat_pad=False``) and, for prompts starting at
position 0, the reference-shaped ``oracle.prefill_attention``.  Tolerances: bf16
attention 1e-2 relative (Frobenius), bf16 layers 2e-2; batching-independence bit exact.
"""

import math

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from pythonintern_b200 import _lib, kernels, workloads  # noqa: E402
from pythonintern_b200.config import KVCacheConfig, ShardConfig  # noqa: E402
from pythonintern_b200.model.kv_cache import PhysicalKVCachePool  # noqa: E402
from pythonintern_b200.model.llama import DistributedLLaMAModel  # noqa: E402
from pythonintern_b200.model.metadata import build_prefill_metadata, prefill_layout  # noqa: E402
from pythonintern_b200.worker.execution_engine import WorkerExecutionEngine  # noqa: E402
from pythonintern_b200.worker.messages import SequenceSlot, StepRequest  # noqa: E402

DEV = torch.device("cuda", 0)


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def to_np(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.check_device_status(DEV, "before test")
    yield
    torch.cuda.synchronize()


def _case(lens, ctx0, nq, nkv, hd, seed, extra_blocks=3):
    """Pool with every sequence's keys at positions 0..ctx0+len-1 behind permuted block tables."""
    bs = 16
    need = [math.ceil((c + L) / bs) for c, L in zip(ctx0, lens)]
    NB = sum(need) + extra_blocks
    gen = torch.Generator().manual_seed(seed)
    perm = torch.randperm(NB, generator=gen).tolist()
    tables, k = [], 0
    for n in need:
        tables.append(perm[k:k + n])
        k += n
    width = max(need)
    tab = np.full((len(lens), width), -1, dtype=np.int32)
    for s, t in enumerate(tables):
        tab[s, :len(t)] = t
    kc = torch.randn(1, NB, bs, nkv, hd, generator=gen).to(torch.bfloat16)
    vc = torch.randn(1, NB, bs, nkv, hd, generator=gen).to(torch.bfloat16)
    q = torch.randn(sum(lens), nq, hd, generator=gen).to(torch.bfloat16)
    return q, kc, vc, tables, tab


def _run(q, kc, vc, tab, lens, ctx0, nq, nkv, hd):
    pos, tidx, ctx, seq_start, last, c0 = prefill_layout(lens, ctx0)
    T = q.shape[0]
    return kernels.prefill_attention(q.view(T, nq * hd).to(DEV), nq, nkv, hd, kc.to(DEV), vc.to(DEV), 0,
                                     torch.from_numpy(tab).to(DEV), torch.from_numpy(seq_start).to(DEV), len(lens),
                                     1 / math.sqrt(hd),
                                     seq_ctx0=None if c0 is None else torch.from_numpy(c0).to(DEV))


def _oracle_rows(q, kc, vc, tables, lens, ctx0):
    """Row r of sequence s: masked attention at position ctx0[s] + t over keys 0..pos."""
    T, nq, hd = q.shape
    nkv = kc.shape[3]
    pool = oracle.KVPool(1, kc.shape[1], 16, nkv, hd)
    pool.k[:] = kc.float().numpy()
    pool.v[:] = vc.float().numpy()
    pos, tidx, _, _, _, _ = prefill_layout(lens, ctx0)
    row_tables = [tables[int(s)] for s in tidx]
    # the token's own K/V are already in the pool: store them again (a no-op)
    knew = np.stack([pool.k[0][row_tables[r][pos[r] // 16], pos[r] % 16] for r in range(T)])
    vnew = np.stack([pool.v[0][row_tables[r][pos[r] // 16], pos[r] % 16] for r in range(T)])
    return oracle.decode_attention(q.float().numpy(), knew, vnew, pos, pool, 0, row_tables, 1 / math.sqrt(hd),
                                   compat_pad=False)


@pytest.mark.parametrize("nq,nkv,hd", [(32, 8, 128), (8, 1, 128), (32, 4, 64), (4, 2, 64), (8, 8, 32),
                                       (16, 2, 128)])
def test_prefill_attention_vs_oracle(nq, nkv, hd):
    lens = [1, 16, 17, 70, 130, 15, 64]
    ctx0 = [0, 0, 5, 0, 33, 16, 0]
    q, kc, vc, tables, tab = _case(lens, ctx0, nq, nkv, hd, seed=nq + hd)
    out = _run(q, kc, vc, tab, lens, ctx0, nq, nkv, hd)
    torch.cuda.synchronize()
    _lib.check_device_status(DEV, "prefill attention")
    want = _oracle_rows(q, kc, vc, tables, lens, ctx0)
    assert rel(to_np(out), want) < 1e-2
    # every row individually, so a wrong row cannot hide in the norm
    got = to_np(out)
    for r in range(got.shape[0]):
        assert rel(got[r], want[r]) < 3e-2, r


def _run_tc(q, kc, vc, tab, lens, ctx0, nq, nkv, hd):
    pos, tidx, ctx, seq_start, last, c0 = prefill_layout(lens, ctx0)
    T = q.shape[0]
    return kernels.prefill_attention(q.view(T, nq * hd).to(DEV), nq, nkv, hd, kc.to(DEV), vc.to(DEV), 0,
                                     torch.from_numpy(tab).to(DEV), torch.from_numpy(seq_start).to(DEV), len(lens),
                                     1 / math.sqrt(hd), tensor_cores=True,
                                     seq_ctx0=None if c0 is None else torch.from_numpy(c0).to(DEV))


@pytest.mark.parametrize("nq,nkv", [(32, 8), (8, 1), (16, 2), (4, 4), (8, 4)])
@pytest.mark.parametrize("lens,ctx0", [([1, 16, 17, 70, 130, 15, 64], [0, 0, 5, 0, 33, 16, 0]),
                                       ([1024, 300, 513], [0, 200, 0])])
def test_prefill_attention_tensor_cores_vs_oracle(nq, nkv, lens, ctx0):
    """The tcgen05 kernel (S and P.V in TMEM, K/V tiles of 64 keys over a 3-stage TMA ring) per
    row against the oracle (the mma.sync kernel keeps head_dim 32 and 64, tested above)."""
    hd = 128
    q, kc, vc, tables, tab = _case(lens, ctx0, nq, nkv, hd, seed=nq * 3 + len(lens))
    out = _run_tc(q, kc, vc, tab, lens, ctx0, nq, nkv, hd)
    torch.cuda.synchronize()
    _lib.check_device_status(DEV, "prefill attention (tensor cores)")
    if sum(lens) > 1000:
        # the oracle's per-row loop is slow: check a spread of rows of every sequence
        rows = sorted({0, 1, 15, 16, 63, 64, 65, 127, 128, 500, 1023, 1024, 1100, 1323, 1324, 1500, sum(lens) - 1})
    else:
        rows = list(range(sum(lens)))
    want = _oracle_rows_subset(q, kc, vc, tables, lens, ctx0, rows)
    got = to_np(out)[rows]
    assert rel(got, want) < 1e-2
    for i, r in enumerate(rows):
        assert rel(got[i], want[i]) < 3e-2, r
    # b2_prefill_attention runs this kernel for head_dim 128: the same bits
    assert torch.equal(out, _run(q, kc, vc, tab, lens, ctx0, nq, nkv, hd))


@pytest.mark.parametrize("nq,nkv", [(32, 8), (8, 1)])
def test_prefill_attention_tensor_cores_rising_scores(nq, nkv):
    """Scores that climb by about 8.7 (log2 units) from one 64-key tile to the next, so the
    kernel's running reference maximum moves on every tile and O is rescaled in TMEM; and
    falling scores, where it never moves and P stays far below 1."""
    hd = 128
    lens, ctx0 = [300, 517], [0, 70]
    for sign in (1.0, -1.0):
        q, kc, vc, tables, tab = _case(lens, ctx0, nq, nkv, hd, seed=nq + 41)
        gen = torch.Generator().manual_seed(5)
        q = (1.0 + 0.05 * torch.randn(q.shape, generator=gen)).to(torch.bfloat16)
        # the key at position t of every sequence: score ~ sign * 6 * (t // 64) + noise
        for s, tb in enumerate(tables):
            for t in range(ctx0[s] + lens[s]):
                blk, off = tb[t // 16], t % 16
                a = sign * 6.0 * (t // 64) / (hd / math.sqrt(hd))
                kc[0, blk, off] = (a + 0.02 * torch.randn(nkv, hd, generator=gen)).to(torch.bfloat16)
        out = _run_tc(q, kc, vc, tab, lens, ctx0, nq, nkv, hd)
        torch.cuda.synchronize()
        _lib.check_device_status(DEV, "prefill attention (tensor cores, rescaling)")
        rows = sorted({0, 1, 63, 64, 65, 128, 200, 299, 300, 301, 400, 555, 700, 816})
        want = _oracle_rows_subset(q, kc, vc, tables, lens, ctx0, rows)
        got = to_np(out)[rows]
        assert np.isfinite(got).all()
        assert rel(got, want) < 1e-2, sign
        for i, r in enumerate(rows):
            assert rel(got[i], want[i]) < 3e-2, (sign, r)


def _oracle_rows_subset(q, kc, vc, tables, lens, ctx0, rows):
    T, nq, hd = q.shape
    nkv = kc.shape[3]
    pool = oracle.KVPool(1, kc.shape[1], 16, nkv, hd)
    pool.k[:] = kc.float().numpy()
    pool.v[:] = vc.float().numpy()
    pos, tidx, _, _, _, _ = prefill_layout(lens, ctx0)
    row_tables = [tables[int(tidx[r])] for r in rows]
    p = pos[rows]
    knew = np.stack([pool.k[0][row_tables[i][p[i] // 16], p[i] % 16] for i in range(len(rows))])
    vnew = np.stack([pool.v[0][row_tables[i][p[i] // 16], p[i] % 16] for i in range(len(rows))])
    return oracle.decode_attention(q.float().numpy()[rows], knew, vnew, p, pool, 0, row_tables, 1 / math.sqrt(hd),
                                   compat_pad=False)


def test_prefill_attention_matches_reference_prefill_shape():
    """ctx0 = 0: the reference's own prefill (oracle.prefill_attention, one sequence per call)."""
    nq, nkv, hd = 32, 8, 128
    lens = [37, 1, 100]
    ctx0 = [0, 0, 0]
    q, kc, vc, tables, tab = _case(lens, ctx0, nq, nkv, hd, seed=3)
    got = to_np(_run(q, kc, vc, tab, lens, None, nq, nkv, hd))
    starts = np.concatenate([[0], np.cumsum(lens)])
    for s, L in enumerate(lens):
        rows = list(range(L))
        k = np.stack([kc[0, tables[s][t // 16], t % 16].float().numpy() for t in rows])[None]
        v = np.stack([vc[0, tables[s][t // 16], t % 16].float().numpy() for t in rows])[None]
        qs = q[starts[s]:starts[s + 1]].float().numpy()[None]
        want = oracle.prefill_attention(qs, k, v, None, 0, None, 1 / math.sqrt(hd))[0]
        assert rel(got[starts[s]:starts[s + 1]], want) < 1e-2


def test_prefill_attention_rows_do_not_depend_on_batching():
    """A sequence's rows are bit-identical whether it runs alone or with others."""
    nq, nkv, hd = 32, 8, 128
    lens = [70, 5, 129, 16]
    ctx0 = [0, 3, 0, 40]
    q, kc, vc, tables, tab = _case(lens, ctx0, nq, nkv, hd, seed=9)
    full = to_np(_run(q, kc, vc, tab, lens, ctx0, nq, nkv, hd))
    starts = np.concatenate([[0], np.cumsum(lens)])
    for s in range(len(lens)):
        one = to_np(_run(q[starts[s]:starts[s + 1]], kc, vc, tab[s:s + 1], [lens[s]], [ctx0[s]], nq, nkv, hd))
        np.testing.assert_array_equal(one, full[starts[s]:starts[s + 1]])


def test_prefill_attention_close_to_per_row_kernel_long_prompts():
    """Prompts of 2048 and 1000 tokens against the per-row paged kernel (pinned separately)."""
    nq, nkv, hd = 32, 8, 128
    lens = [2048, 1000, 3]
    ctx0 = [0, 0, 0]
    q, kc, vc, tables, tab = _case(lens, ctx0, nq, nkv, hd, seed=17)
    got = _run(q, kc, vc, tab, lens, None, nq, nkv, hd)
    pos, tidx, ctx, _, _, _ = prefill_layout(lens)
    T = q.shape[0]
    ref = kernels.paged_attention(q.view(T, -1).to(DEV), nq, nkv, hd, kc.to(DEV), vc.to(DEV), 0,
                                  torch.from_numpy(tab).to(DEV), torch.from_numpy(tidx).to(DEV),
                                  torch.from_numpy(ctx).to(DEV), False, 1 / math.sqrt(hd))
    torch.cuda.synchronize()
    _lib.check_device_status(DEV, "prefill attention")
    assert rel(to_np(got), to_np(ref)) < 1e-2


def test_prefill_attention_bad_block_is_reported():
    nq, nkv, hd = 4, 1, 32
    kc = torch.zeros(1, 4, 16, nkv, hd, device=DEV, dtype=torch.bfloat16)
    tab = torch.tensor([[0, 9]], dtype=torch.int32, device=DEV)  # 9 is not a block of a 4-block pool
    kernels.prefill_attention(torch.zeros(20, nq * hd, device=DEV, dtype=torch.bfloat16), nq, nkv, hd, kc, kc, 0,
                              tab, torch.tensor([0, 20], dtype=torch.int32, device=DEV), 1, 0.1)
    with pytest.raises(IndexError):
        _lib.check_device_status(DEV, "prefill attention")


def test_prefill_attention_table_too_short_is_reported():
    nq, nkv, hd = 4, 1, 32
    kc = torch.zeros(1, 4, 16, nkv, hd, device=DEV, dtype=torch.bfloat16)
    tab = torch.tensor([[2]], dtype=torch.int32, device=DEV)  # 20 tokens need two blocks
    kernels.prefill_attention(torch.zeros(20, nq * hd, device=DEV, dtype=torch.bfloat16), nq, nkv, hd, kc, kc, 0,
                              tab, torch.tensor([0, 20], dtype=torch.int32, device=DEV), 1, 0.1)
    with pytest.raises(IndexError):
        _lib.check_device_status(DEV, "prefill attention")


def test_prefill_attention_rejects_float32():
    kc = torch.zeros(1, 4, 16, 1, 32, device=DEV)
    with pytest.raises(_lib.B2Error):
        kernels.prefill_attention(torch.zeros(4, 128, device=DEV), 4, 1, 32, kc, kc, 0,
                                  torch.zeros(1, 1, dtype=torch.int32, device=DEV),
                                  torch.tensor([0, 4], dtype=torch.int32, device=DEV), 1, 0.1)


# ------------------------------------------------------------------ the batched prefill forward
def test_varlen_prefill_model_vs_oracle():
    """One forward over five prompts of different lengths == the oracle's per-prompt forwards."""
    cfg = workloads.llama3_8b_config(num_layers=1, max_seq_len=512)
    cfg.vocab_size = 4096
    sd = workloads.synthetic_state_dict(cfg, seed=21)
    model = DistributedLLaMAModel(cfg, device=DEV)
    model.load_state_dict(sd)
    nb = 64
    pool = PhysicalKVCachePool(nb, 16, cfg.num_kv_heads, cfg.head_dim, cfg.num_layers, DEV, "bfloat16")
    ocfg = oracle.OracleConfig(cfg.vocab_size, cfg.hidden_dim, cfg.num_layers, cfg.num_heads, cfg.num_kv_heads,
                               cfg.intermediate_dim, cfg.max_seq_len, cfg.rms_norm_eps)
    om = oracle.OracleModel(ocfg, [{k: v.float().numpy() for k, v in sd.items()}],
                            [oracle.KVPool(cfg.num_layers, nb, 16, cfg.num_kv_heads, cfg.head_dim)])
    gen = torch.Generator().manual_seed(22)
    lens = [150, 17, 1, 64, 33]
    perm = torch.randperm(nb, generator=gen).tolist()
    tables, k = [], 0
    for P in lens:
        n = math.ceil(P / 16)
        tables.append(perm[k:k + n])
        k += n
    toks = [torch.randint(0, cfg.vocab_size, (P,), generator=gen) for P in lens]
    md = build_prefill_metadata(lens, tables, DEV)
    ids = torch.cat(toks)[None].to(DEV)
    tr = []
    logits = model(ids, None, pool, tables, True, 0, metadata=md, trace=tr)
    tok, top = model.greedy(ids, None, pool, tables, True, 0, metadata=build_prefill_metadata(lens, tables, DEV))
    torch.cuda.synchronize()
    _lib.check_device_status(DEV, "varlen prefill")
    otr_all, olg_all = [], []
    for s, P in enumerate(lens):
        otr = []
        olg = om.forward(toks[s].numpy()[None], np.arange(P)[None], [tables[s]], True, trace=otr)
        otr_all.append(otr)
        olg_all.append(olg[0])
    for layer in range(cfg.num_layers):
        want = np.concatenate([otr[layer][0] for otr in otr_all])
        assert rel(tr[layer].cpu().numpy(), want) < 2e-2
    assert rel(to_np(logits), np.stack(olg_all)) < 2e-2
    np.testing.assert_array_equal(tok.cpu().numpy(), torch.argmax(logits, dim=-1).cpu().numpy())
    np.testing.assert_allclose(to_np(top), to_np(logits[:, :10]), rtol=0, atol=0)


def test_engine_batched_prefill_matches_per_sequence_prefill():
    """execute_step with the prompts in one forward vs one forward per prompt (the reference's loop)."""
    cfg = workloads.tinyllama_config(num_layers=2)
    cfg.vocab_size = 4096
    sd = workloads.synthetic_state_dict(cfg, seed=31)
    gen = torch.Generator().manual_seed(32)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=gen).tolist() for n in (20, 45, 1, 33, 16)]
    res = []
    for batched in (False, True):
        eng = WorkerExecutionEngine(cfg, ShardConfig(0, 1), KVCacheConfig(16, 128, str(DEV)), None, DEV,
                                    batch_prefills=batched)
        eng.model.load_state_dict(sd)
        ids = [f"s{i}" for i in range(len(prompts))]
        for sid, p in zip(ids, prompts):
            eng.kv_manager.allocate_blocks_for_sequence(sid, len(p))
        resp = eng.execute_step(StepRequest(0, [SequenceSlot(sid, True, p, 0, len(p),
                                                             list(eng.kv_manager.block_tables[sid].physical_block_ids))
                                                for sid, p in zip(ids, prompts)]))
        assert [t.seq_id for t in resp.sampled_tokens] == ids
        res.append(np.asarray([t.top_logits for t in resp.sampled_tokens]))
        # the KV the prefill stored must be the same too: compare the pools' used blocks
        res.append(eng.kv_manager.pool.k_cache.float().cpu().numpy())
    assert rel(res[2], res[0]) < 2e-2
    assert rel(res[3], res[1]) < 2e-2


def test_engine_prefill_groups_respect_the_token_cap():
    cfg = workloads.tinyllama_config(num_layers=1)
    cfg.vocab_size = 1024
    eng = WorkerExecutionEngine(cfg, ShardConfig(0, 1), KVCacheConfig(16, 64, str(DEV)), None, DEV,
                                max_prefill_tokens=100)

    class S:
        def __init__(self, n):
            self.prompt_token_ids = [0] * n

    groups = eng._prefill_groups([S(60), S(30), S(20), S(150), S(5)])
    assert [[len(s.prompt_token_ids) for s in g] for g in groups] == [[60, 30], [20], [150], [5]]
