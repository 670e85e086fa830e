// C-ABI entry points of the linear layers.  bf16 runs on the tcgen05 kernel
// (gemm_tc.cu), float32 on the FFMA kernel (gemm_simt.cu).
#include "gemm.cuh"

namespace b2 {

static int check_common(const void* x, int M, int K, int N, int dtype, int y_dtype, const char* who) {
  B2_CHECK_ARG(M >= 0 && K > 0 && N > 0, "%s: bad sizes M=%d K=%d N=%d", who, M, K, N);
  B2_CHECK_ARG(valid_dtype(dtype) && valid_dtype(y_dtype), "%s: bad dtype", who);
  B2_CHECK_ARG(M == 0 || x, "%s: null input", who);
  return B2_OK;
}

}  // namespace b2

extern "C" {

size_t b2_linear_workspace_bytes(int M, int N, int K, int dtype) {
  if (dtype != B2_BF16 || M <= 0 || N <= 0 || K <= 0) return 0;
  size_t a = b2::gemm_tc_workspace_bytes(M, N, K, b2::kEpiStore);
  size_t b = b2::gemm_tc_workspace_bytes(M, N, K, b2::kEpiSwiglu);
  return a > b ? a : b;
}

int b2_linear(const void* x, int64_t ldx, int M, int K, const void* w, int N, const float* bias,
              void* y, int64_t ldy, int dtype, int y_dtype, void* workspace, size_t workspace_bytes,
              int32_t* status, b2_stream_t stream) {
  int rc = b2::check_common(x, M, K, N, dtype, y_dtype, "b2_linear");
  if (rc) return rc;
  B2_CHECK_ARG(ldx >= K && ldy >= N, "b2_linear: row strides too small");
  if (M == 0) return B2_OK;
  B2_CHECK_ARG(w && y, "b2_linear: null pointer");
  if (dtype == B2_F32) return b2::gemm_simt(x, ldx, M, K, w, nullptr, N, bias, y, ldy, dtype, y_dtype, stream);
  b2::GemmSeg seg{w, N, 0};
  return b2::gemm_tc(x, ldx, M, K, &seg, 1, b2::kEpiStore, bias, y, ldy, y_dtype, workspace, workspace_bytes,
                     status, stream);
}

int b2_linear_qkv(const void* x, int64_t ldx, int M, int K, const void* wq, int Nq, const void* wk,
                  int Nk, const void* wv, int Nv, void* y, int64_t ldy, int dtype, void* workspace,
                  size_t workspace_bytes, int32_t* status, b2_stream_t stream) {
  int rc = b2::check_common(x, M, K, Nq + Nk + Nv, dtype, dtype, "b2_linear_qkv");
  if (rc) return rc;
  B2_CHECK_ARG(Nq > 0 && Nk > 0 && Nv > 0, "b2_linear_qkv: bad segment sizes");
  B2_CHECK_ARG(ldx >= K && ldy >= (int64_t)Nq + Nk + Nv, "b2_linear_qkv: row strides too small");
  if (M == 0) return B2_OK;
  B2_CHECK_ARG(wq && wk && wv && y, "b2_linear_qkv: null pointer");
  const size_t esz = b2::dtype_bytes(dtype);
  if (dtype == B2_F32) {
    char* yb = static_cast<char*>(y);
    rc = b2::gemm_simt(x, ldx, M, K, wq, nullptr, Nq, nullptr, yb, ldy, dtype, dtype, stream);
    if (rc) return rc;
    rc = b2::gemm_simt(x, ldx, M, K, wk, nullptr, Nk, nullptr, yb + esz * Nq, ldy, dtype, dtype, stream);
    if (rc) return rc;
    return b2::gemm_simt(x, ldx, M, K, wv, nullptr, Nv, nullptr, yb + esz * (Nq + Nk), ldy, dtype, dtype, stream);
  }
  b2::GemmSeg segs[3] = {{wq, Nq, 0}, {wk, Nk, Nq}, {wv, Nv, Nq + Nk}};
  return b2::gemm_tc(x, ldx, M, K, segs, 3, b2::kEpiStore, nullptr, y, ldy, dtype, workspace, workspace_bytes,
                     status, stream);
}

int b2_linear_swiglu(const void* x, int64_t ldx, int M, int K, const void* w_gate, const void* w_up,
                     int N, void* y, int64_t ldy, int dtype, void* workspace,
                     size_t workspace_bytes, int32_t* status, b2_stream_t stream) {
  int rc = b2::check_common(x, M, K, N, dtype, dtype, "b2_linear_swiglu");
  if (rc) return rc;
  B2_CHECK_ARG(ldx >= K && ldy >= N, "b2_linear_swiglu: row strides too small");
  if (M == 0) return B2_OK;
  B2_CHECK_ARG(w_gate && w_up && y, "b2_linear_swiglu: null pointer");
  if (dtype == B2_F32) return b2::gemm_simt(x, ldx, M, K, w_gate, w_up, N, nullptr, y, ldy, dtype, dtype, stream);
  b2::GemmSeg segs[2] = {{w_gate, N, 0}, {w_up, N, 0}};
  return b2::gemm_tc(x, ldx, M, K, segs, 2, b2::kEpiSwiglu, nullptr, y, ldy, dtype, workspace, workspace_bytes,
                     status, stream);
}

int b2_linear_residual_norm(const void* x, int64_t ldx, int M, int K, const void* w, int N, float* h, int64_t ldh,
                            const float* norm_w, void* z, int64_t ldz, float* ss, void* workspace,
                            size_t workspace_bytes, int32_t* status, b2_stream_t stream) {
  int rc = b2::check_common(x, M, K, N, B2_BF16, B2_BF16, "b2_linear_residual_norm");
  if (rc) return rc;
  B2_CHECK_ARG(ldx >= K && ldh >= N && ldz >= N, "b2_linear_residual_norm: row strides too small");
  if (M == 0) return B2_OK;
  B2_CHECK_ARG(w && h && norm_w && z && ss, "b2_linear_residual_norm: null pointer");
  if (M > 512 || N % 128 != 0)
    return b2::fail(B2_ENOTSUP, "b2_linear_residual_norm: needs M <= 512 and N %% 128 == 0 (M=%d N=%d)", M, N);
  b2::GemmSeg seg{w, N, 0};
  b2::RowNorm rn{};
  rn.res_h = h;
  rn.ldh = ldh;
  rn.norm_w = norm_w;
  rn.z = z;
  rn.ldz = ldz;
  rn.ss_out = ss;
  return b2::gemm_tc(x, ldx, M, K, &seg, 1, b2::kEpiStore, nullptr, nullptr, N, B2_BF16, workspace, workspace_bytes,
                     status, stream, nullptr, &rn);
}

int b2_linear_qkv_rownorm(const void* x, int64_t ldx, int M, int K, const void* wq, int Nq, const void* wk, int Nk,
                          const void* wv, int Nv, void* y, int64_t ldy, const float* ss, int n_ss, int dim, float eps,
                          void* workspace, size_t workspace_bytes, int32_t* status, b2_stream_t stream) {
  int rc = b2::check_common(x, M, K, Nq + Nk + Nv, B2_BF16, B2_BF16, "b2_linear_qkv_rownorm");
  if (rc) return rc;
  B2_CHECK_ARG(Nq > 0 && Nk > 0 && Nv > 0 && n_ss > 0 && dim > 0, "b2_linear_qkv_rownorm: bad sizes");
  B2_CHECK_ARG(ldx >= K && ldy >= (int64_t)Nq + Nk + Nv, "b2_linear_qkv_rownorm: row strides too small");
  if (M == 0) return B2_OK;
  B2_CHECK_ARG(wq && wk && wv && y && ss, "b2_linear_qkv_rownorm: null pointer");
  b2::GemmSeg segs[3] = {{wq, Nq, 0}, {wk, Nk, Nq}, {wv, Nv, Nq + Nk}};
  b2::RowNorm rn{};
  rn.row_ss = ss;
  rn.n_ss = n_ss;
  rn.ss_scale = 1.f / (float)dim;
  rn.ss_eps = eps;
  return b2::gemm_tc(x, ldx, M, K, segs, 3, b2::kEpiStore, nullptr, y, ldy, B2_BF16, workspace, workspace_bytes,
                     status, stream, nullptr, &rn);
}

int b2_linear_swiglu_rownorm(const void* x, int64_t ldx, int M, int K, const void* w_gate, const void* w_up, int N,
                             void* y, int64_t ldy, const float* ss, int n_ss, int dim, float eps, void* workspace,
                             size_t workspace_bytes, int32_t* status, b2_stream_t stream) {
  int rc = b2::check_common(x, M, K, N, B2_BF16, B2_BF16, "b2_linear_swiglu_rownorm");
  if (rc) return rc;
  B2_CHECK_ARG(n_ss > 0 && dim > 0, "b2_linear_swiglu_rownorm: bad sizes");
  B2_CHECK_ARG(ldx >= K && ldy >= N, "b2_linear_swiglu_rownorm: row strides too small");
  if (M == 0) return B2_OK;
  B2_CHECK_ARG(w_gate && w_up && y && ss, "b2_linear_swiglu_rownorm: null pointer");
  b2::GemmSeg segs[2] = {{w_gate, N, 0}, {w_up, N, 0}};
  b2::RowNorm rn{};
  rn.row_ss = ss;
  rn.n_ss = n_ss;
  rn.ss_scale = 1.f / (float)dim;
  rn.ss_eps = eps;
  return b2::gemm_tc(x, ldx, M, K, segs, 2, b2::kEpiSwiglu, nullptr, y, ldy, B2_BF16, workspace, workspace_bytes,
                     status, stream, nullptr, &rn);
}

int b2_linear_qkv_rope_kv(const void* x, int64_t ldx, int M, int K, const void* wq, const void* wk, const void* wv,
                          int nq, int nkv, int head_dim, const float* ss, int n_ss, int dim, float eps,
                          const int64_t* rope_pos, const int64_t* store_pos, const int32_t* table_index,
                          const int32_t* block_tables, int table_stride, int num_blocks, int block_size,
                          const float* cos, const float* sin, int max_seq_len, void* q_out, void* k_cache,
                          void* v_cache, int layer, void* workspace, size_t workspace_bytes, int32_t* status,
                          b2_stream_t stream) {
  int rc = b2::check_common(x, M, K, (nq + 2 * nkv) * head_dim, B2_BF16, B2_BF16, "b2_linear_qkv_rope_kv");
  if (rc) return rc;
  B2_CHECK_ARG(nq > 0 && nkv > 0 && ldx >= K, "b2_linear_qkv_rope_kv: bad sizes");
  B2_CHECK_ARG(num_blocks > 0 && block_size > 0 && table_stride > 0 && layer >= 0 && max_seq_len > 0,
               "b2_linear_qkv_rope_kv: bad cache geometry");
  if (M == 0) return B2_OK;
  if (head_dim != 128 || M > 512)
    return b2::fail(B2_ENOTSUP, "b2_linear_qkv_rope_kv: needs head_dim 128 and at most 512 rows");
  B2_CHECK_ARG(wq && wk && wv && rope_pos && block_tables && cos && sin && q_out && k_cache && v_cache,
               "b2_linear_qkv_rope_kv: null pointer");
  B2_CHECK_ARG(!ss || (n_ss > 0 && dim > 0), "b2_linear_qkv_rope_kv: bad row-norm sizes");
  b2::GemmSeg segs[3] = {{wq, nq * head_dim, 0}, {wk, nkv * head_dim, nq * head_dim},
                         {wv, nkv * head_dim, (nq + nkv) * head_dim}};
  b2::RowNorm rn{};
  if (ss) {
    rn.row_ss = ss;
    rn.n_ss = n_ss;
    rn.ss_scale = 1.f / (float)dim;
    rn.ss_eps = eps;
  }
  b2::RopeKV rk{};
  rk.nq = nq;
  rk.nkv = nkv;
  rk.rope_pos = rope_pos;
  rk.store_pos = store_pos;
  rk.table_index = table_index;
  rk.tables = block_tables;
  rk.table_stride = table_stride;
  rk.num_blocks = num_blocks;
  rk.block_size = block_size;
  rk.max_seq_len = max_seq_len;
  rk.cos_t = cos;
  rk.sin_t = sin;
  rk.q_out = q_out;
  rk.k_cache = k_cache;
  rk.v_cache = v_cache;
  rk.layer_off = (int64_t)num_blocks * block_size * nkv * head_dim * layer;
  return b2::gemm_tc(x, ldx, M, K, segs, 3, b2::kEpiStore, nullptr, nullptr, (nq + 2 * nkv) * head_dim, B2_BF16,
                     workspace, workspace_bytes, status, stream, nullptr, ss ? &rn : nullptr, &rk);
}

}  // extern "C"
