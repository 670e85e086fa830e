"""Kernel-level parity of libb2tp against the numpy oracle (GPU).

Each test calls one C-ABI entry point through pythonintern_b200.kernels on seeded
inputs and compares with the oracle restatement of the reference function it
replaces.  Tolerances: float32 kernels 1e-5 relative (the reference's float32 bar),
bf16 kernels 2e-2 relative (Frobenius), integer/index work bit exact.
"""

import math

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from pythonintern_b200 import _lib, kernels  # noqa: E402
from pythonintern_b200.model.attention import RotaryEmbedding  # noqa: E402

DEV = torch.device("cuda", 0)


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def g(seed):
    return torch.Generator().manual_seed(seed)


def to_np(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.check_device_status(DEV, "before test")
    yield
    torch.cuda.synchronize()


# ------------------------------------------------------------------ RMSNorm / embedding / argmax
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,dim", [(1, 64), (7, 256), (33, 4096)])
def test_rmsnorm_residual(dtype, rows, dim):
    x = torch.randn(rows, dim, generator=g(rows)) * 3
    r = torch.randn(rows, dim, generator=g(rows + 1))
    w = torch.rand(dim, generator=g(2)) + 0.5
    h = r.clone().to(DEV)
    y = kernels.rmsnorm(x.to(DEV, dtype), w.to(DEV), 1e-5, residual=h, h_out=h, out_dtype=dtype)
    xr = x.to(dtype).float().numpy() + r.numpy()
    want = oracle.rmsnorm(xr, w.numpy(), 1e-5)
    tol = 1e-6 if dtype == torch.float32 else 8e-3
    assert rel(to_np(h), xr) < 1e-7
    assert rel(to_np(y), want) < tol


def test_rmsnorm_plain_float32_matches_reference_formula():
    x = torch.randn(5, 64, generator=g(9))
    w = torch.rand(64, generator=g(10)) + 0.5
    y = kernels.rmsnorm(x.to(DEV), w.to(DEV), 1e-5)
    ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-5) * w  # layers.py:182-184 in torch fp32
    assert rel(to_np(y), ref.numpy()) < 1e-6


def test_embedding_and_range_error():
    table = torch.randn(50, 32, generator=g(1)).to(DEV, torch.bfloat16)
    ids = torch.tensor([0, 49, 7, 7], device=DEV)
    out = kernels.embedding(ids, table, out_dtype=torch.float32)
    assert torch.equal(out, table[ids].float())
    kernels.embedding(torch.tensor([50], device=DEV), table)
    with pytest.raises(IndexError):
        _lib.check_device_status(DEV, "embedding")


def test_argmax_first_max_like_torch():
    x = torch.randn(9, 1000, generator=g(3))
    x[2, 10] = x[2, 500] = 100.0  # tie -> first index
    x[4] = -float("inf")
    out = kernels.argmax(x.to(DEV))
    assert out.cpu().tolist() == torch.argmax(x, dim=-1).tolist()


# ------------------------------------------------------------------ linears
def _linear_case(M, N, K, dtype, seed):
    x = torch.randn(M, K, generator=g(seed))
    w = torch.randn(N, K, generator=g(seed + 1)) / math.sqrt(K)
    xd, wd = x.to(DEV, dtype), w.to(DEV, dtype)
    return xd, wd, xd.float().cpu().numpy(), wd.float().cpu().numpy()


@pytest.mark.parametrize("M,N,K", [(1, 64, 32), (8, 256, 256), (40, 688, 256), (5, 256, 688), (130, 96, 344)])
def test_linear_float32(M, N, K):
    xd, wd, x, w = _linear_case(M, N, K, torch.float32, M * 7 + N)
    y = kernels.linear(xd, wd)
    assert rel(to_np(y), oracle.column_parallel_linear(x, w.T)) < 1e-6


@pytest.mark.parametrize("M,N,K", [
    (1, 128, 64), (1, 4096, 4096), (7, 384, 512), (16, 256, 2048), (33, 1024, 1024), (64, 512, 5632),
    (128, 6144, 4096), (129, 256, 256), (200, 384, 320), (300, 640, 2048), (1, 4096, 14336),
    (128, 14336, 4096), (100, 12800, 1024), (64, 10240, 2048),  # 74..147 tiles: one wave, idle SMs
    (240, 768, 4096), (240, 4096, 14336), (512, 4096, 7168), (513, 512, 1024),  # 128-wide token tiles to 512
    # the 8B layer's GEMMs at eight ranks: q|k|v 768 x 4096 (split-K 8, one k block per stage
    # set), o_proj 4096 x 512 (two k blocks per split), down 4096 x 1792
    (128, 768, 4096), (128, 4096, 512), (128, 4096, 1792), (8, 4096, 512),
])
def test_linear_bf16_tensor_cores(M, N, K):
    """tcgen05 GEMM (swap-AB, split-K where chosen) against the float64 oracle on the same bf16 inputs."""
    xd, wd, x, w = _linear_case(M, N, K, torch.bfloat16, M * 13 + K)
    y = kernels.linear(xd, wd, out_dtype=torch.float32)
    torch.cuda.synchronize()
    _lib.check_device_status(DEV, "linear")
    want = x @ w.T
    assert rel(to_np(y), want) < 3e-5  # float32 accumulation of exact bf16 products
    yb = kernels.linear(xd, wd)  # bf16 output rounding
    assert rel(to_np(yb), want) < 8e-3


def test_linear_bf16_repeat_reuses_workspace():
    xd, wd, x, w = _linear_case(4, 4096, 14336, torch.bfloat16, 5)
    ys = [to_np(kernels.linear(xd, wd, out_dtype=torch.float32)) for _ in range(3)]
    assert np.array_equal(ys[0], ys[1]) and np.array_equal(ys[1], ys[2])
    assert rel(ys[0], x @ w.T) < 1e-5


def test_linear_bias_and_strided_rows():
    xd, wd, x, w = _linear_case(12, 256, 128, torch.bfloat16, 11)
    bias = torch.randn(256, generator=g(4))
    y = kernels.linear(xd[::3], wd, bias=bias.to(DEV), out_dtype=torch.float32)
    assert rel(to_np(y), x[::3] @ w.T + bias.numpy()) < 1e-5
    xf, wf, x32, w32 = _linear_case(12, 64, 32, torch.float32, 12)
    y = kernels.linear(xf[1::4], wf)
    assert rel(to_np(y), x32[1::4] @ w32.T) < 1e-6


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M", [1, 19, 128])
def test_linear_qkv(dtype, M):
    K, Nq, Nk = 512, 512, 128
    x = torch.randn(M, K, generator=g(M)).to(DEV, dtype)
    ws = [(torch.randn(n, K, generator=g(n + M)) / math.sqrt(K)).to(DEV, dtype) for n in (Nq, Nk, Nk)]
    y = kernels.linear_qkv(x, *ws)
    xn = to_np(x)
    want = np.concatenate([xn @ to_np(w).T for w in ws], axis=1)
    assert rel(to_np(y), want) < (1e-6 if dtype == torch.float32 else 8e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(1, 344, 256), (8, 2816, 2048), (128, 1792, 4096), (70, 200, 256),
                                   (128, 14336, 4096), (16, 12288, 1024), (300, 2816, 2048), (1000, 1792, 1024),
                                   # 74..147 tiles of 128 rows: one shorter tile per SM (97, 88, 68 rows;
                                   # the last tile of the two ragged shapes is partial)
                                   (128, 13000, 1024), (40, 10000, 512)])
def test_linear_swiglu(dtype, M, N, K):
    x = torch.randn(M, K, generator=g(M)).to(DEV, dtype)
    wg = (torch.randn(N, K, generator=g(1)) / math.sqrt(K)).to(DEV, dtype)
    wu = (torch.randn(N, K, generator=g(2)) / math.sqrt(K)).to(DEV, dtype)
    y = kernels.linear_swiglu(x, wg, wu)
    xn = to_np(x)
    want = oracle.silu(xn @ to_np(wg).T) * (xn @ to_np(wu).T)
    assert rel(to_np(y), want) < (1e-5 if dtype == torch.float32 else 8e-3)


def test_large_gemm_repeated_calls_are_identical():
    """The 8B gate|up shape (112 tiles) and a plain GEMM over the same weight, called back
    to back and interleaved: results agree bit for bit between calls."""
    M, N, K = 128, 14336, 4096
    x = torch.randn(M, K, generator=g(7)).to(DEV, torch.bfloat16)
    wg = (torch.randn(N, K, generator=g(8)) / math.sqrt(K)).to(DEV, torch.bfloat16)
    wu = (torch.randn(N, K, generator=g(9)) / math.sqrt(K)).to(DEV, torch.bfloat16)
    y1 = kernels.linear_swiglu(x, wg, wu)
    y2 = kernels.linear(x, wg)
    y3 = kernels.linear_swiglu(x, wg, wu)
    y4 = kernels.linear(x, wg)
    torch.cuda.synchronize()
    _lib.check_device_status(DEV, "large GEMM")
    assert torch.equal(y1, y3) and torch.equal(y2, y4)
    assert rel(to_np(y2), to_np(x) @ to_np(wg).T) < 8e-3


@pytest.mark.parametrize("M", [128, 5, 240])
def test_deferred_rmsnorm_producer_and_consumers(M):
    """Row-parallel GEMM + residual add leaving z = h * w and per-tile sums of h^2, then
    q|k|v and SwiGLU GEMMs that apply the RMS scale per row: against float64 on the same
    bf16 inputs (the normalised GEMM input is never rounded, so compare the scaled GEMM
    of z, and the explicit rmsnorm + GEMM path at the bf16 tolerance)."""
    H, K, I, eps = 4096, 4096, 1024, 1e-5
    x = torch.randn(M, K, generator=g(M + 1)).to(DEV, torch.bfloat16)
    w = (torch.randn(H, K, generator=g(M + 2)) / math.sqrt(K)).to(DEV, torch.bfloat16)
    h0 = torch.randn(M, H, generator=g(M + 3)).to(DEV)
    nw = (1.0 + 0.1 * torch.randn(H, generator=g(M + 4))).to(DEV)
    h = h0.clone()
    z = torch.empty(M, H, dtype=torch.bfloat16, device=DEV)
    ss = torch.empty(M, H // 128, device=DEV)
    assert kernels.linear_residual_norm(x, w, h, nw, z, ss)
    torch.cuda.synchronize()
    _lib.check_device_status(DEV, "residual norm")
    h_ref = to_np(h0) + to_np(x) @ to_np(w).T
    assert rel(to_np(h), h_ref) < 3e-5
    assert rel(to_np(z), h_ref * to_np(nw)) < 8e-3
    assert rel(to_np(ss), (h_ref.reshape(M, H // 128, 128) ** 2).sum(-1)) < 1e-4
    inv = 1.0 / np.sqrt((to_np(ss).sum(-1) / H) + eps)
    wg = (torch.randn(I, H, generator=g(M + 5)) / math.sqrt(H)).to(DEV, torch.bfloat16)
    wu = (torch.randn(I, H, generator=g(M + 6)) / math.sqrt(H)).to(DEV, torch.bfloat16)
    y = kernels.linear_swiglu_rownorm(z, wg, wu, ss, eps)
    zn = to_np(z)
    want = oracle.silu(inv[:, None] * (zn @ to_np(wg).T)) * (inv[:, None] * (zn @ to_np(wu).T))
    assert rel(to_np(y), want) < 8e-3
    xn = kernels.rmsnorm(h, nw, eps, out_dtype=torch.bfloat16)  # the unfused path
    assert rel(to_np(y), to_np(kernels.linear_swiglu(xn, wg, wu))) < 2e-2
    wq, wk, wv = [(torch.randn(n, H, generator=g(M + 7 + i)) / math.sqrt(H)).to(DEV, torch.bfloat16)
                  for i, n in enumerate((512, 128, 128))]
    q = kernels.linear_qkv_rownorm(z, wq, wk, wv, ss, eps)
    want = inv[:, None] * (zn @ np.concatenate([to_np(wq), to_np(wk), to_np(wv)]).T)
    assert rel(to_np(q), want) < 8e-3


@pytest.mark.parametrize("M,nq,nkv,rownorm", [(128, 32, 8, False), (128, 4, 1, True), (7, 8, 2, True),
                                               (240, 4, 1, True), (300, 8, 2, False)])
def test_fused_qkv_rope_kv_is_bit_identical(M, nq, nkv, rownorm):
    """q|k|v GEMM with RoPE and the paged KV write in its epilogue equals the GEMM followed
    by rope_kv_write, bit for bit: q, and every K/V slot of the pool."""
    hd, K, bs, L, eps = 128, 1024, 16, 2, 1e-5
    x = torch.randn(M, K, generator=g(M + 11)).to(DEV, torch.bfloat16)
    wq, wk, wv = [(torch.randn(n * hd, K, generator=g(M + 12 + i)) / math.sqrt(K)).to(DEV, torch.bfloat16)
                  for i, n in enumerate((nq, nkv, nkv))]
    NB = M * 4 + 3
    tables = torch.randperm(NB - 3, generator=g(5))[: M * 4].view(M, 4).to(torch.int32).to(DEV)
    pos = torch.randint(0, 4 * bs, (M,), generator=g(6)).to(DEV)
    tab_cos = torch.randn(512, hd, generator=g(7)).to(DEV)
    tab_sin = torch.randn(512, hd, generator=g(8)).to(DEV)
    ss = torch.rand(M, K // 128, generator=g(9)).to(DEV) * 50 if rownorm else None
    outs = []
    for fused in (True, False):
        kc = torch.zeros(L, NB, bs, nkv, hd, dtype=torch.bfloat16, device=DEV)
        vc = torch.zeros_like(kc)
        q = torch.empty(M, nq * hd, dtype=torch.bfloat16, device=DEV)
        if fused:
            assert kernels.linear_qkv_rope_kv(x, wq, wk, wv, nq, nkv, hd, pos, None, None, tables, tab_cos,
                                              tab_sin, q, kc, vc, 1, row_ss=ss, eps=eps)
        else:
            qkv = kernels.linear_qkv_rownorm(x, wq, wk, wv, ss, eps) if rownorm else kernels.linear_qkv(x, wq, wk, wv)
            kernels.rope_kv_write(qkv, nq, nkv, hd, pos, None, None, tables, tab_cos, tab_sin, q, kc, vc, 1)
        torch.cuda.synchronize()
        _lib.check_device_status(DEV, "qkv rope")
        outs.append((q, kc, vc))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_fused_qkv_rope_kv_declines_shapes_without_a_cluster_plan():
    """240 rows of the 8B TP=1 q|k|v (96 output tiles) get no split-K cluster plan: the fused
    call launches nothing and says so, and the caller's two-call path runs instead."""
    M, hd, K = 240, 128, 4096
    x = torch.randn(M, K, generator=g(3)).to(DEV, torch.bfloat16)
    wq, wk, wv = [torch.zeros(n * hd, K, dtype=torch.bfloat16, device=DEV) for n in (32, 8, 8)]
    kc = torch.zeros(1, 64, 16, 8, hd, dtype=torch.bfloat16, device=DEV)
    q = torch.empty(M, 32 * hd, dtype=torch.bfloat16, device=DEV)
    tables = torch.zeros(M, 1, dtype=torch.int32, device=DEV)
    pos = torch.zeros(M, dtype=torch.int64, device=DEV)
    tab = torch.zeros(16, hd, device=DEV)
    assert not kernels.linear_qkv_rope_kv(x, wq, wk, wv, 32, 8, hd, pos, None, None, tables, tab, tab, q, kc,
                                          kc.clone(), 0)


def test_split_k_workspace_shared_across_shapes():
    """Launches with different tile counts share one workspace; none may read another's partials."""
    shapes = [(3, 5632, 2048, "swiglu"), (37, 2560, 2048, "linear"), (64, 256, 8192, "linear"),
              (3, 256, 4096, "linear"), (150, 14336, 4096, "swiglu"), (2, 4096, 14336, "linear"),
              (37, 2560, 2048, "linear"), (1, 128, 4096, "linear")]
    for i, (M, N, K, kind) in enumerate(shapes):
        x = torch.randn(M, K, generator=g(i)).to(DEV, torch.bfloat16)
        w = (torch.randn(N, K, generator=g(i + 50)) / math.sqrt(K)).to(DEV, torch.bfloat16)
        xn, wn = to_np(x), to_np(w)
        if kind == "swiglu":
            u = (torch.randn(N, K, generator=g(i + 90)) / math.sqrt(K)).to(DEV, torch.bfloat16)
            y = kernels.linear_swiglu(x, w, u)
            want = oracle.silu(xn @ wn.T) * (xn @ to_np(u).T)
        else:
            y = kernels.linear(x, w)
            want = xn @ wn.T
        assert rel(to_np(y), want) < 8e-3, (M, N, K, kind)


# ------------------------------------------------------------------ RoPE + paged KV write
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rope_kv_write_slots_bit_exact(dtype):
    nq, nkv, hd, NB, bs, L = 4, 2, 32, 12, 16, 3
    n = 20
    qkv = torch.randn(n, (nq + 2 * nkv) * hd, generator=g(5)).to(DEV, dtype)
    pos = torch.tensor([0, 1, 15, 16, 17, 31, 32, 47, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 40, 41])
    tables = torch.tensor([[7, 3, 10, 0]], dtype=torch.int32)
    tidx = torch.zeros(n, dtype=torch.int32)
    rope = RotaryEmbedding(hd, 128, 10000.0, DEV)
    kc = torch.zeros(L, NB, bs, nkv, hd, device=DEV, dtype=dtype)
    vc = torch.zeros_like(kc)
    q = torch.empty(n, nq * hd, device=DEV, dtype=dtype)
    kernels.rope_kv_write(qkv, nq, nkv, hd, pos.to(DEV), None, tidx.to(DEV), tables.to(DEV), rope.cos_cached,
                          rope.sin_cached, q, kc, vc, layer=1)
    torch.cuda.synchronize()
    _lib.check_device_status(DEV, "rope")
    x = qkv.float().cpu().view(n, nq + 2 * nkv, hd)
    cos, sin = rope.cos_cached.cpu(), rope.sin_cached.cpu()
    # torch float32 rotate-half, two roundings (attention.py:58-63)
    c, s = cos[pos].unsqueeze(1), sin[pos].unsqueeze(1)
    xr = torch.cat((-x[..., hd // 2:], x[..., :hd // 2]), dim=-1)
    rot = (x * c) + (xr * s)
    kc_h, vc_h = kc.float().cpu(), vc.float().cpu()
    for i in range(n):
        blk, off = oracle.physical_slot([7, 3, 10, 0], int(pos[i]), bs)
        assert torch.equal(vc_h[1, blk, off], x[i, nq + nkv:])  # values: exact copy
        want_k = rot[i, nq:nq + nkv].to(dtype).float()
        assert torch.equal(kc_h[1, blk, off], want_k)
    assert torch.equal(q.float().cpu().view(n, nq, hd), rot[:, :nq].to(dtype).float())
    assert kc_h[0].abs().sum() == 0 and kc_h[2].abs().sum() == 0  # other layers untouched


def test_rope_kv_write_out_of_range_is_reported():
    nq, nkv, hd = 2, 1, 32
    qkv = torch.randn(2, (nq + 2 * nkv) * hd, device=DEV)
    rope = RotaryEmbedding(hd, 64, 10000.0, DEV)
    kc = torch.zeros(1, 4, 16, nkv, hd, device=DEV)
    q = torch.empty(2, nq * hd, device=DEV)
    tables = torch.tensor([[1, 2]], dtype=torch.int32, device=DEV)
    # position 40 needs block index 2, past the 2-entry table (the reference raises IndexError)
    kernels.rope_kv_write(qkv, nq, nkv, hd, torch.tensor([3, 40], device=DEV), None,
                          torch.zeros(2, dtype=torch.int32, device=DEV), tables, rope.cos_cached, rope.sin_cached,
                          q, kc, kc.clone(), 0)
    with pytest.raises(IndexError):
        _lib.check_device_status(DEV, "rope")


# ------------------------------------------------------------------ paged attention
def _attn_case(dtype, B, nq, nkv, hd, ctxs, NB=None, seed=0):
    bs = 16
    nblk = [math.ceil(c / bs) for c in ctxs]
    NB = NB or sum(nblk) + 3
    gen = g(seed)
    perm = torch.randperm(NB, generator=gen).tolist()
    tables, k = [], 0
    for n in nblk:
        tables.append(perm[k:k + n])
        k += n
    width = max(nblk)
    tab = np.full((B, width), -1, dtype=np.int32)
    for b, t in enumerate(tables):
        tab[b, :len(t)] = t
    kc = torch.randn(1, NB, bs, nkv, hd, generator=gen).to(dtype)
    vc = torch.randn(1, NB, bs, nkv, hd, generator=gen).to(dtype)
    q = torch.randn(B, nq, hd, generator=gen).to(dtype)
    return q, kc, vc, tables, tab


def _oracle_attn(q, kc, vc, tables, ctxs, compat):
    B, nq, hd = q.shape
    nkv = kc.shape[3]
    pool = oracle.KVPool(1, kc.shape[1], 16, nkv, hd)
    pool.k[:] = kc.float().numpy()
    pool.v[:] = vc.float().numpy()
    # store the "new" token as the value already in the cache, so the store is a no-op
    pos = [c - 1 for c in ctxs]
    knew = np.stack([pool.k[0][tables[b][pos[b] // 16], pos[b] % 16] for b in range(B)])
    vnew = np.stack([pool.v[0][tables[b][pos[b] // 16], pos[b] % 16] for b in range(B)])
    return oracle.decode_attention(q.float().numpy(), knew, vnew, pos, pool, 0, tables, 1 / math.sqrt(hd), compat)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("nq,nkv,hd", [(8, 2, 32), (4, 4, 64), (32, 4, 64), (32, 8, 128), (4, 1, 128), (16, 8, 128)])
@pytest.mark.parametrize("compat", [True, False])
@pytest.mark.parametrize("splits", [1, 3])
def test_paged_attention(dtype, nq, nkv, hd, compat, splits):
    ctxs = [1, 17, 40, 16, 100]
    B = len(ctxs)
    q, kc, vc, tables, tab = _attn_case(dtype, B, nq, nkv, hd, ctxs, seed=nq + hd + splits)
    out = kernels.paged_attention(q.view(B, nq * hd).to(DEV), nq, nkv, hd, kc.to(DEV), vc.to(DEV), 0,
                                  torch.from_numpy(tab).to(DEV), None,
                                  torch.tensor(ctxs, dtype=torch.int32, device=DEV), compat, 1 / math.sqrt(hd),
                                  num_splits=splits)
    torch.cuda.synchronize()
    _lib.check_device_status(DEV, "attention")
    want = _oracle_attn(q, kc, vc, tables, ctxs, compat)
    assert rel(to_np(out), want) < (1e-5 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("splits", [1, 4, 16])
def test_paged_attention_long_context_bf16(splits):
    ctxs = [2048, 1500, 2049, 33]
    B, nq, nkv, hd = len(ctxs), 32, 8, 128
    q, kc, vc, tables, tab = _attn_case(torch.bfloat16, B, nq, nkv, hd, ctxs, seed=splits)
    out = kernels.paged_attention(q.view(B, -1).to(DEV), nq, nkv, hd, kc.to(DEV), vc.to(DEV), 0,
                                  torch.from_numpy(tab).to(DEV), None,
                                  torch.tensor(ctxs, dtype=torch.int32, device=DEV), True, 1 / math.sqrt(hd),
                                  num_splits=splits)
    want = _oracle_attn(q, kc, vc, tables, ctxs, True)
    assert rel(to_np(out), want) < 1e-2


def test_paged_attention_split_workspace_reuse_deterministic():
    ctxs = [300, 5, 77]
    B, nq, nkv, hd = 3, 8, 2, 64
    q, kc, vc, tables, tab = _attn_case(torch.bfloat16, B, nq, nkv, hd, ctxs, seed=4)
    args = (q.view(B, -1).to(DEV), nq, nkv, hd, kc.to(DEV), vc.to(DEV), 0, torch.from_numpy(tab).to(DEV), None,
            torch.tensor(ctxs, dtype=torch.int32, device=DEV), True, 1 / math.sqrt(hd))
    outs = [to_np(kernels.paged_attention(*args, num_splits=5)) for _ in range(3)]
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


def test_paged_attention_bad_block_is_reported():
    B, nq, nkv, hd = 1, 4, 1, 32
    kc = torch.zeros(1, 4, 16, nkv, hd, device=DEV)
    tab = torch.tensor([[0, 9]], dtype=torch.int32, device=DEV)  # 9 is not a block of a 4-block pool
    kernels.paged_attention(torch.zeros(1, nq * hd, device=DEV), nq, nkv, hd, kc, kc, 0, tab, None,
                            torch.tensor([20], dtype=torch.int32, device=DEV), True, 0.1)
    with pytest.raises(IndexError):
        _lib.check_device_status(DEV, "attention")
