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


def _case(seed):
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
    kc = torch.randn(2, NB, bs, nkv, hd, generator=gen).to(DEV)
    vc = torch.randn(2, NB, bs, nkv, hd, generator=gen).to(DEV)
    q = torch.randn(B, nq * hd, generator=gen).to(DEV)
    return q, kc, vc, torch.from_numpy(tab).to(DEV), torch.tensor(ctxs, dtype=torch.int32, device=DEV), nq, nkv, hd


def _noalloc(q, kc, vc, tab, ctx, nq, nkv, hd, splits, out):
    NB, bs = kc.shape[1], kc.shape[2]
    return _lib.lib().b2_paged_attention_noalloc(
        q.data_ptr(), q.stride(0), q.shape[0], nq, nkv, hd, kc.data_ptr(), vc.data_ptr(), 1, NB, bs,
        tab.data_ptr(), tab.shape[1], None, ctx.data_ptr(), 1, 1.0 / math.sqrt(hd), out.data_ptr(), out.stride(0),
        _lib.B2_F32, splits, _lib.status_ptr(DEV), _lib.stream_ptr(DEV))


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


def test_noalloc_rejects_calls_beyond_its_scratch():
    q, kc, vc, tab, ctx, nq, nkv, hd = _case(1)
    out = torch.empty_like(q)
    # 6 rows x 32 heads x 1024 splits x 128 dims x 4 bytes is far beyond the static array
    rc = _noalloc(q, kc, vc, tab, ctx, nq, nkv, hd, 1024, out)
    assert rc == _lib.B2_EINVAL
    assert "static array holds" in _lib.last_error()
