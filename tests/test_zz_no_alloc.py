"""The allocation-free paged-attention entry point, called through the C ABI.

b2_paged_attention_noalloc serves callers that cannot allocate device memory (a
host reaching the library only through the plain C ABI, with no device allocator
of its own, or a worker whose device memory belongs to another runtime's pool).
It must give the same result as b2_paged_attention with a caller workspace, call
after call, although its split scratch is one static array shared by every call.

This file is collected last on purpose: if it fails, a run that stops at the first
failure has already run every other test.  It passes alone in a fresh process
(where its first call also performs the one-time scratch lookup) and after the
other tests.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from pythonintern_b200 import _lib, kernels  # noqa: E402

DEV = torch.device("cuda", 0)


def _case(seed, dtype=torch.float32):
    gen = torch.Generator().manual_seed(seed)
    B, nq, nkv, hd, bs = 6, 32, 8, 128, 16
    ctxs = [700, 1, 333, 64, 1024, 129]
    nblk = [math.ceil(c / bs) for c in ctxs]
    NB = sum(nblk) + 5
    perm = torch.randperm(NB, generator=gen).tolist()
    tab = np.full((B, max(nblk)), -1, dtype=np.int32)
    k = 0
    for b, n in enumerate(nblk):
        tab[b, :n] = perm[k:k + n]
        k += n
    kc = torch.randn(2, NB, bs, nkv, hd, generator=gen).to(dtype).to(DEV)
    vc = torch.randn(2, NB, bs, nkv, hd, generator=gen).to(dtype).to(DEV)
    q = torch.randn(B, nq * hd, generator=gen).to(dtype).to(DEV)
    return q, kc, vc, torch.from_numpy(tab).to(DEV), torch.tensor(ctxs, dtype=torch.int32, device=DEV), nq, nkv, hd


def _noalloc(q, kc, vc, tab, ctx, nq, nkv, hd, splits, out):
    NB, bs = kc.shape[1], kc.shape[2]
    return _lib.lib().b2_paged_attention_noalloc(
        q.data_ptr(), q.stride(0), q.shape[0], nq, nkv, hd, kc.data_ptr(), vc.data_ptr(), 1, NB, bs,
        tab.data_ptr(), tab.shape[1], None, ctx.data_ptr(), 1, 1.0 / math.sqrt(hd), out.data_ptr(), out.stride(0),
        _lib.B2_BF16 if q.dtype == torch.bfloat16 else _lib.B2_F32, splits, _lib.status_ptr(DEV),
        _lib.stream_ptr(DEV))


def _torch_reference(q, kc, vc, tab, ctx, nq, nkv, hd):
    """float32 decode attention of layer 1 with the reference's unmasked zero padding: every row
    also counts (max_ctx - ctx) zero scores in its softmax denominator (attention.py:190-224)."""
    q, kc, vc = q.float().cpu(), kc.float().cpu(), vc.float().cpu()
    tab, ctx = tab.cpu(), ctx.cpu().tolist()
    L = max(ctx)
    rep = nq // nkv
    out = torch.zeros(q.shape[0], nq * hd)
    for b, c in enumerate(ctx):
        ids = [int(t) for t in tab[b][: (c + 15) // 16]]
        k = kc[1, ids].reshape(-1, nkv, hd)[:c]
        v = vc[1, ids].reshape(-1, nkv, hd)[:c]
        for h in range(nq):
            s = (k[:, h // rep] @ q[b, h * hd:(h + 1) * hd]) / math.sqrt(hd)
            s = torch.cat([s, torch.zeros(L - c)])
            p = torch.softmax(s, 0)[:c]
            out[b, h * hd:(h + 1) * hd] = p @ v[:, h // rep]
    return out


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("splits", [4, 7])
def test_noalloc_matches_workspace_entry_point_twice(splits):
    q, kc, vc, tab, ctx, nq, nkv, hd = _case(splits)
    want = kernels.paged_attention(q, nq, nkv, hd, kc, vc, 1, tab, None, ctx, True, 1.0 / math.sqrt(hd),
                                   num_splits=splits)
    for _ in range(2):  # the second call sees the first call's leftovers in the shared scratch
        out = torch.full_like(want, float("nan"))
        rc = _noalloc(q, kc, vc, tab, ctx, nq, nkv, hd, splits, out)
        assert rc == _lib.B2_OK, _lib.last_error()
        torch.cuda.synchronize()
        _lib.check_device_status(DEV, "noalloc attention")
        assert rel(out, want) < 1e-5  # the float32 attention tolerance of test_kernels_gpu.py


def test_noalloc_bf16_split_path_against_torch_and_allocates_nothing():
    """The bf16 path the model runs (tensor-core kernel, block size 16) with splits > 1:
    bit-identical to the workspace entry point, within the bf16 attention tolerance of an
    independent float32 torch computation, on two calls in a row, and neither torch's
    allocator nor the device's free memory moves across those calls (the first call on the
    device, made before the measurement, may load the library's module)."""
    splits = 5
    q, kc, vc, tab, ctx, nq, nkv, hd = _case(9, torch.bfloat16)
    want_ws = kernels.paged_attention(q, nq, nkv, hd, kc, vc, 1, tab, None, ctx, True, 1.0 / math.sqrt(hd),
                                      num_splits=splits)
    want = _torch_reference(q, kc, vc, tab, ctx, nq, nkv, hd)
    outs = [torch.full_like(want_ws, float("nan")) for _ in range(3)]
    assert _noalloc(q, kc, vc, tab, ctx, nq, nkv, hd, splits, outs[0]) == _lib.B2_OK, _lib.last_error()
    torch.cuda.synchronize()
    alloc0 = torch.cuda.memory_allocated(DEV)
    free0 = torch.cuda.mem_get_info(DEV)[0]
    for out in outs[1:]:
        rc = _noalloc(q, kc, vc, tab, ctx, nq, nkv, hd, splits, out)
        assert rc == _lib.B2_OK, _lib.last_error()
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated(DEV) == alloc0
    assert torch.cuda.mem_get_info(DEV)[0] == free0
    _lib.check_device_status(DEV, "noalloc attention bf16")
    for out in outs:
        assert torch.equal(out, want_ws)
        assert rel(out, want) < 1e-2  # the bf16 attention tolerance of test_kernels_gpu.py


def test_noalloc_rejects_bad_arguments():
    """Bad arguments are rejected with the same checks as b2_paged_attention (the entry point
    runs them before it clears any shared counter, so a rejected call cannot disturb a call
    still running on another stream)."""
    q, kc, vc, tab, ctx, nq, nkv, hd = _case(2)
    out = torch.empty_like(q)
    bad_rows = 70000  # over the 65535-row limit: rejected by the argument checks
    rc = _lib.lib().b2_paged_attention_noalloc(
        q.data_ptr(), q.stride(0), bad_rows, nq, nkv, hd, kc.data_ptr(), vc.data_ptr(), 1, kc.shape[1], 16,
        tab.data_ptr(), tab.shape[1], None, ctx.data_ptr(), 1, 0.1, out.data_ptr(), out.stride(0), _lib.B2_F32, 4,
        _lib.status_ptr(DEV), _lib.stream_ptr(DEV))
    assert rc == _lib.B2_EINVAL and "65535" in _lib.last_error()


def test_noalloc_rejects_calls_beyond_its_scratch():
    q, kc, vc, tab, ctx, nq, nkv, hd = _case(1)
    out = torch.empty_like(q)
    # 6 rows x 32 heads x 1024 splits x 128 dims x 4 bytes is far beyond the static array
    rc = _noalloc(q, kc, vc, tab, ctx, nq, nkv, hd, 1024, out)
    assert rc == _lib.B2_EINVAL
    assert "static array holds" in _lib.last_error()
