"""Tensor-level wrappers around the libb2tp entry points.

Each function validates its tensors (CUDA, dtype, contiguity), passes raw device
pointers and the current CUDA stream to the C ABI and returns the output tensor.
Device-side range errors are collected in a per-device status word; call
``_lib.check_device_status(device)`` at a synchronisation point to surface them.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from pythonintern_b200 import _lib
from pythonintern_b200._lib import check, dtype_code, ptr, require_cuda, status_ptr, stream_ptr

SM_COUNT_DEFAULT = 148


def _sms(device) -> int:
    try:
        return torch.cuda.get_device_properties(device).multi_processor_count
    except Exception:  # pragma: no cover
        return SM_COUNT_DEFAULT


def _c(t: torch.Tensor, name: str) -> torch.Tensor:
    require_cuda(t, name)
    return t if t.is_contiguous() else t.contiguous()


def embedding(ids: torch.Tensor, table: torch.Tensor, out_dtype: Optional[torch.dtype] = None,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``table[ids]`` (engine/model/llama.py:150).  ids: int64 [n]."""
    ids = _c(ids.reshape(-1).to(torch.int64), "ids")
    table = _c(table, "table")
    od = out_dtype or table.dtype
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=od, device=table.device)
    check(_lib.lib().b2_embedding(ptr(ids), ids.numel(), ptr(table), table.shape[0], table.shape[1],
                                  dtype_code(table.dtype), ptr(out), dtype_code(out.dtype),
                                  status_ptr(table.device), stream_ptr(table.device)), "b2_embedding")
    return out


def residual_add(x: torch.Tensor, h: torch.Tensor):
    """In-place ``h += x`` on the float32 residual stream (engine/model/llama.py:70,75)."""
    require_cuda(x, "x")
    dim = x.shape[-1]
    x2 = _c(x, "x").reshape(-1, dim)
    assert h.is_contiguous() and h.numel() == x2.numel()
    check(_lib.lib().b2_rmsnorm(ptr(x2), dtype_code(x2.dtype), ptr(h), dtype_code(h.dtype), ptr(h),
                                dtype_code(h.dtype), None, 0.0, None, 0, x2.shape[0], dim,
                                stream_ptr(x.device)), "b2_rmsnorm")


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
            h_out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``h = x (+ residual)``; ``h_out = h``; returns ``h * rsqrt(mean(h^2) + eps) * weight``.

    (engine/tensor_parallel/layers.py:179-184).  Rows are the leading dimensions.
    """
    require_cuda(x, "x")
    dim = x.shape[-1]
    x2 = _c(x, "x").reshape(-1, dim)
    rows = x2.shape[0]
    w = _c(weight.to(torch.float32), "weight")
    if residual is not None:
        residual = _c(residual, "residual").reshape(-1, dim)
    if h_out is not None:
        assert h_out.is_contiguous() and h_out.numel() == x2.numel()
    od = out_dtype or x.dtype
    if out is None:
        out = torch.empty(x.shape, dtype=od, device=x.device)
    check(_lib.lib().b2_rmsnorm(ptr(x2), dtype_code(x2.dtype), ptr(residual),
                                dtype_code(residual.dtype) if residual is not None else 0, ptr(h_out),
                                dtype_code(h_out.dtype) if h_out is not None else 0, ptr(w), float(eps),
                                ptr(out), dtype_code(out.dtype), rows, dim, stream_ptr(x.device)), "b2_rmsnorm")
    return out


def _linear_ws(device, M, N, K, dtype_c):
    nbytes = _lib.lib().b2_linear_workspace_bytes(M, N, K, dtype_c)
    ws = _lib.workspace(device, "linear", nbytes)
    return ws, nbytes


def linear(x: torch.Tensor, w_packed: torch.Tensor, bias: Optional[torch.Tensor] = None,
           out_dtype: Optional[torch.dtype] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x @ w_packed.T (+ bias)`` with ``w_packed`` the [N, K] (K-contiguous) weight.

    ColumnParallelLinear.forward / RowParallelLinear partial GEMM
    (engine/tensor_parallel/layers.py:78-86, :147-152).
    """
    require_cuda(x, "x")
    K = x.shape[-1]
    if x.dim() == 2 and x.stride(1) == 1 and x.stride(0) >= K:
        x2 = x  # row-strided 2D input (e.g. the last token of every sequence)
    else:
        x2 = _c(x, "x").reshape(-1, K)
    M = x2.shape[0]
    N = w_packed.shape[0]
    assert w_packed.shape[1] == K and w_packed.is_contiguous()
    dc = dtype_code(w_packed.dtype)
    if x2.dtype != w_packed.dtype:
        x2 = x2.to(w_packed.dtype)
    od = out_dtype or w_packed.dtype
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=od, device=x.device)
    b = None if bias is None else _c(bias.to(torch.float32), "bias")
    ws, nbytes = _linear_ws(x.device, M, N, K, dc)
    check(_lib.lib().b2_linear(ptr(x2), x2.stride(0), M, K, ptr(w_packed), N, ptr(b), ptr(out), N, dc, dtype_code(od),
                               ptr(ws), nbytes, status_ptr(x.device), stream_ptr(x.device)), "b2_linear")
    return out


def linear_qkv(x: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Concatenated ``[x Wq^T | x Wk^T | x Wv^T]`` (engine/model/attention.py:156-158)."""
    K = x.shape[-1]
    x2 = _c(x, "x").reshape(-1, K)
    M = x2.shape[0]
    Nq, Nk, Nv = wq.shape[0], wk.shape[0], wv.shape[0]
    dc = dtype_code(wq.dtype)
    if x2.dtype != wq.dtype:
        x2 = x2.to(wq.dtype)
    if out is None:
        out = torch.empty(M, Nq + Nk + Nv, dtype=wq.dtype, device=x.device)
    ws, nbytes = _linear_ws(x.device, M, Nq + Nk + Nv, K, dc)
    check(_lib.lib().b2_linear_qkv(ptr(x2), K, M, K, ptr(wq), Nq, ptr(wk), Nk, ptr(wv), Nv, ptr(out),
                                   out.stride(0), dc, ptr(ws), nbytes, status_ptr(x.device),
                                   stream_ptr(x.device)), "b2_linear_qkv")
    return out


def linear_swiglu(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``silu(x Wg^T) * (x Wu^T)`` (engine/model/mlp.py:80-82)."""
    K = x.shape[-1]
    x2 = _c(x, "x").reshape(-1, K)
    M = x2.shape[0]
    N = w_gate.shape[0]
    dc = dtype_code(w_gate.dtype)
    if x2.dtype != w_gate.dtype:
        x2 = x2.to(w_gate.dtype)
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=w_gate.dtype, device=x.device)
    ws, nbytes = _linear_ws(x.device, M, N, K, dc)
    check(_lib.lib().b2_linear_swiglu(ptr(x2), K, M, K, ptr(w_gate), ptr(w_up), N, ptr(out), N, dc, ptr(ws),
                                      nbytes, status_ptr(x.device), stream_ptr(x.device)), "b2_linear_swiglu")
    return out


def linear_residual_norm(x: torch.Tensor, w_packed: torch.Tensor, h: torch.Tensor, norm_w: torch.Tensor,
                         z: torch.Tensor, ss: torch.Tensor) -> bool:
    """Deferred-RMSNorm producer at world size 1: ``h += x @ w^T``; ``z = bf16(h * norm_w)``;
    ``ss[m, t]`` = sum of h[m]^2 over 128-column tile t.

    RowParallelLinear partial GEMM + residual add + the sums the next RMSNorm needs
    (layers.py:147-162, 179-184; llama.py:70-75).  Returns False, having launched
    nothing, when the shape gets no split-K cluster plan (too many 128-row output tiles,
    or more than 512 rows).
    """
    require_cuda(x, "x")
    K = x.shape[-1]
    x2 = x if (x.dim() == 2 and x.stride(1) == 1) else _c(x, "x").reshape(-1, K)
    M, N = x2.shape[0], w_packed.shape[0]
    if x2.dtype != torch.bfloat16 or w_packed.dtype != torch.bfloat16:
        return False
    ws, nbytes = _linear_ws(x.device, M, N, K, _lib.B2_BF16)
    rc = _lib.lib().b2_linear_residual_norm(ptr(x2), x2.stride(0), M, K, ptr(w_packed), N, ptr(h), h.stride(0),
                                            ptr(norm_w), ptr(z), z.stride(0), ptr(ss), ptr(ws), nbytes,
                                            status_ptr(x.device), stream_ptr(x.device))
    if rc == _lib.B2_ENOTSUP:
        return False
    check(rc, "b2_linear_residual_norm")
    return True


def linear_qkv_rownorm(z: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, ss: torch.Tensor,
                       eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``linear_qkv`` of the RMS-normalised rows: z = bf16(h * w) and ss from
    ``linear_residual_norm``; each output row is scaled by rsqrt(sum(ss) / hidden + eps)."""
    M, K = z.shape
    Nq, Nk, Nv = wq.shape[0], wk.shape[0], wv.shape[0]
    if out is None:
        out = torch.empty(M, Nq + Nk + Nv, dtype=wq.dtype, device=z.device)
    ws, nbytes = _linear_ws(z.device, M, Nq + Nk + Nv, K, _lib.B2_BF16)
    check(_lib.lib().b2_linear_qkv_rownorm(ptr(z), z.stride(0), M, K, ptr(wq), Nq, ptr(wk), Nk, ptr(wv), Nv,
                                           ptr(out), out.stride(0), ptr(ss), ss.shape[1], K, float(eps), ptr(ws),
                                           nbytes, status_ptr(z.device), stream_ptr(z.device)),
          "b2_linear_qkv_rownorm")
    return out


def linear_swiglu_rownorm(z: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, ss: torch.Tensor, eps: float,
                          out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``linear_swiglu`` of the RMS-normalised rows (see ``linear_qkv_rownorm``)."""
    M, K = z.shape
    N = w_gate.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=w_gate.dtype, device=z.device)
    ws, nbytes = _linear_ws(z.device, M, N, K, _lib.B2_BF16)
    check(_lib.lib().b2_linear_swiglu_rownorm(ptr(z), z.stride(0), M, K, ptr(w_gate), ptr(w_up), N, ptr(out),
                                              out.stride(0), ptr(ss), ss.shape[1], K, float(eps), ptr(ws), nbytes,
                                              status_ptr(z.device), stream_ptr(z.device)),
          "b2_linear_swiglu_rownorm")
    return out


def linear_qkv_rope_kv(x: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, nq: int, nkv: int,
                       head_dim: int, rope_pos: torch.Tensor, store_pos: Optional[torch.Tensor],
                       table_index: Optional[torch.Tensor], block_tables: torch.Tensor, cos: torch.Tensor,
                       sin: torch.Tensor, q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                       layer: int, row_ss: Optional[torch.Tensor] = None, eps: float = 1e-5) -> bool:
    """``linear_qkv`` (or ``linear_qkv_rownorm`` with ``row_ss``) + ``rope_kv_write`` in one
    launch, bit-identical to the two.  Returns False, having launched nothing, when the
    shape has no fused form (head_dim != 128, more than 512 rows, or no cluster plan)."""
    M, K = x.shape
    if x.dtype != torch.bfloat16 or head_dim != 128 or M > 512:
        return False
    _, NB, bs, ckv, chd = k_cache.shape
    assert ckv == nkv and chd == head_dim, "cache geometry does not match the heads"
    assert block_tables.dtype == torch.int32 and block_tables.is_contiguous()
    N = (nq + 2 * nkv) * head_dim
    ws, nbytes = _linear_ws(x.device, M, N, K, _lib.B2_BF16)
    rc = _lib.lib().b2_linear_qkv_rope_kv(
        ptr(x), x.stride(0), M, K, ptr(wq), ptr(wk), ptr(wv), nq, nkv, head_dim, ptr(row_ss),
        row_ss.shape[1] if row_ss is not None else 0, K, float(eps), ptr(rope_pos), ptr(store_pos),
        ptr(table_index), ptr(block_tables), block_tables.shape[1], NB, bs, ptr(cos), ptr(sin), cos.shape[0],
        ptr(q_out), ptr(k_cache), ptr(v_cache), layer, ptr(ws), nbytes, status_ptr(x.device), stream_ptr(x.device))
    if rc == _lib.B2_ENOTSUP:
        return False
    check(rc, "b2_linear_qkv_rope_kv")
    return True


def rope_kv_write(qkv: torch.Tensor, nq: int, nkv: int, head_dim: int, rope_pos: torch.Tensor,
                  store_pos: Optional[torch.Tensor], table_index: Optional[torch.Tensor],
                  block_tables: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, q_out: torch.Tensor,
                  k_cache: torch.Tensor, v_cache: torch.Tensor, layer: int):
    """RoPE on q/k and the paged KV write (engine/model/attention.py:46-63, :166-184)."""
    n = qkv.shape[0]
    _, NB, bs, ckv, chd = k_cache.shape
    assert ckv == nkv and chd == head_dim, "cache geometry does not match the heads"
    assert block_tables.dtype == torch.int32 and block_tables.is_contiguous()
    check(_lib.lib().b2_rope_kv_write(
        ptr(qkv), qkv.stride(0), n, nq, nkv, head_dim, ptr(rope_pos), ptr(store_pos), ptr(table_index),
        ptr(block_tables), block_tables.shape[1], NB, bs, ptr(cos), ptr(sin), cos.shape[0], ptr(q_out),
        ptr(k_cache), ptr(v_cache), layer, dtype_code(qkv.dtype), status_ptr(qkv.device),
        stream_ptr(qkv.device)), "b2_rope_kv_write")


def attention_splits(n_rows: int, nkv: int, max_ctx: int, block_size: int = 16, device=None) -> int:
    """KV split count: as many splits as keep every (row, kv head, split) CTA in ONE wave
    (two attention CTAs are resident per SM), with at least 4 KV blocks per split; with
    fewer (row, kv head) pairs than SMs, at most one CTA per SM and 4 splits.

    A second, partly filled wave leaves HBM idle at the tail (measured on B200 at context
    2048, batch 128: one kv head per row, 5 splits over 2.2 waves took 40 us, 2 splits in
    one wave 30 us; two kv heads per row, 3 splits 61 us, 1 split 45 us).  The context is
    counted in buckets of 32 blocks, the block-table width a captured decode graph is
    sized for, so an eager call and a graph replay over the same sequences pick the
    same split count and give bit-identical results.
    """
    sms = _sms(device) if device is not None else SM_COUNT_DEFAULT
    slots = 2 * sms
    pairs = max(1, n_rows * nkv)
    if pairs >= slots:
        return 1
    nblk = 32 * max(1, math.ceil(max_ctx / (32 * block_size)))
    if pairs < sms:
        # at most one CTA per SM, where the kernel runs 8-warp CTAs; measured on B200 at
        # context 2048: one kv head x 128 rows best with 1 split (26 us; 2 splits of 4-warp
        # CTAs 30 us), 32 rows and a single row with 4 (11-12 us; 9 and 32 splits 17-25 us)
        return max(1, min(sms // pairs, 4, max(1, nblk // 8)))
    s = min(slots // pairs, max(1, nblk // 4), 256)
    return max(1, s)


def paged_attention(q: torch.Tensor, nq: int, nkv: int, head_dim: int, k_cache: torch.Tensor,
                    v_cache: torch.Tensor, layer: int, block_tables: torch.Tensor,
                    table_index: Optional[torch.Tensor], ctx_lens: torch.Tensor, compat_pad: bool,
                    scale: float, out: Optional[torch.Tensor] = None, num_splits: int = 1) -> torch.Tensor:
    """Paged GQA attention, one query token per row (engine/model/attention.py:175-228)."""
    n_rows = q.shape[0]
    _, NB, bs, _, _ = k_cache.shape
    if out is None:
        out = torch.empty(n_rows, nq * head_dim, dtype=q.dtype, device=q.device)
    nbytes = _lib.lib().b2_paged_attention_workspace_bytes(n_rows, nq, nkv, head_dim, num_splits)
    ws = _lib.workspace(q.device, "attention", nbytes)
    check(_lib.lib().b2_paged_attention(
        ptr(q), q.stride(0), n_rows, nq, nkv, head_dim, ptr(k_cache), ptr(v_cache), layer, NB, bs,
        ptr(block_tables), block_tables.shape[1], ptr(table_index), ptr(ctx_lens), 1 if compat_pad else 0,
        float(scale), ptr(out), out.stride(0), dtype_code(q.dtype), ptr(ws), nbytes, num_splits,
        status_ptr(q.device), stream_ptr(q.device)), "b2_paged_attention")
    return out


def prefill_supported(dtype: torch.dtype, nq: int, nkv: int, head_dim: int, block_size: int) -> bool:
    """Shapes ``b2_prefill_attention`` runs (the per-row ``paged_attention`` covers the rest)."""
    return (dtype == torch.bfloat16 and block_size == 16 and head_dim in (32, 64, 128)
            and nq % nkv == 0 and nq // nkv in (1, 2, 4, 8))


def prefill_attention(q: torch.Tensor, nq: int, nkv: int, head_dim: int, k_cache: torch.Tensor,
                      v_cache: torch.Tensor, layer: int, block_tables: torch.Tensor, seq_start: torch.Tensor,
                      n_seqs: int, scale: float, seq_ctx0: Optional[torch.Tensor] = None,
                      out: Optional[torch.Tensor] = None, tensor_cores: bool = False) -> torch.Tensor:
    """Causal attention of every prompt token of ``n_seqs`` sequences in one launch.

    Rows ``[seq_start[s], seq_start[s+1])`` of ``q`` are sequence s at positions
    ``seq_ctx0[s] + (row - seq_start[s])``; each attends to keys ``0..pos`` of its own
    sequence in the pool (block-table row s).  engine/model/attention.py:166-174,211-228,
    which the reference runs one sequence at a time (execution_engine.py:85-111).
    ``tensor_cores`` calls the tcgen05 kernel directly (head_dim 128).
    """
    n_rows = q.shape[0]
    _, NB, bs, _, _ = k_cache.shape
    if out is None:
        out = torch.empty(n_rows, nq * head_dim, dtype=q.dtype, device=q.device)
    assert seq_start.dtype == torch.int32 and seq_start.numel() >= n_seqs + 1
    assert seq_ctx0 is None or (seq_ctx0.dtype == torch.int32 and seq_ctx0.numel() >= n_seqs)
    name = "b2_prefill_attention_tc" if tensor_cores else "b2_prefill_attention"
    check(getattr(_lib.lib(), name)(
        ptr(q), q.stride(0), n_rows, nq, nkv, head_dim, ptr(k_cache), ptr(v_cache), layer, NB, bs,
        ptr(block_tables), block_tables.shape[1], ptr(seq_start), ptr(seq_ctx0), n_seqs, float(scale),
        ptr(out), out.stride(0), dtype_code(q.dtype), status_ptr(q.device), stream_ptr(q.device)), name)
    return out


def argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """First index of each row's maximum (engine/worker/execution_engine.py:103,133)."""
    assert logits.dtype == torch.float32 and logits.dim() == 2 and logits.stride(1) == 1
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    check(_lib.lib().b2_argmax(ptr(logits), logits.stride(0), logits.shape[0], logits.shape[1], ptr(out),
                               stream_ptr(logits.device)), "b2_argmax")
    return out
