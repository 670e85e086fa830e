// Embedding gather, residual add + RMSNorm, and greedy argmax.
//
// These are HBM-bound row kernels: one CTA per row, 16-byte accesses where the
// row allows it, statistics in float32.
#include "common.cuh"

namespace b2 {

// ---------------------------------------------------------------- embedding
// out[i, :] = table[ids[i], :]   (engine/model/llama.py:150)
__global__ void embedding_kernel(const int64_t* __restrict__ ids, const void* __restrict__ table,
                                 int vocab, int dim, int dtype, void* __restrict__ out,
                                 int out_dtype, int32_t* status) {
  const int row = blockIdx.x;
  const int64_t id = ids[row];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) raise_status(status, B2_DEV_RANGE);
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    float v = ok ? ld_dyn(table, dtype, (size_t)id * dim + c) : 0.f;
    st_dyn(out, out_dtype, (size_t)row * dim + c, v);
  }
}

// ---------------------------------------------------------------- RMSNorm
// h = x (+ res); h_out = h; y = h * rsqrt(mean(h^2) + eps) * w
// (engine/tensor_parallel/layers.py:179-184).  The row is staged in shared memory
// as float32 so x/res/h_out may alias (each element is read before it is written
// by the same thread).
__global__ void rmsnorm_kernel(const void* x, int x_dtype, const void* res, int res_dtype,
                               void* h_out, int h_dtype, const float* __restrict__ w, float eps,
                               void* y, int y_dtype, int dim) {
  extern __shared__ float srow[];
  __shared__ float red[32];
  const size_t base = (size_t)blockIdx.x * dim;
  float ss = 0.f;
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    float v = ld_dyn(x, x_dtype, base + c);
    if (res) v += ld_dyn(res, res_dtype, base + c);
    srow[c] = v;
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)dim + eps);
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    const float v = srow[c];
    if (h_out) st_dyn(h_out, h_dtype, base + c, v);
    if (y) st_dyn(y, y_dtype, base + c, v * inv * w[c]);
  }
}

// ---------------------------------------------------------------- argmax
// First index of the row maximum, like torch.argmax (execution_engine.py:103,133).
__global__ void argmax_kernel(const float* __restrict__ logits, int64_t ld, int cols,
                              int64_t* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const float* row = logits + (size_t)blockIdx.x * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const float v = row[c];
    if (v > best || (v == best && c < bi) || (v != v && best == best)) {  // NaN wins, like torch
      best = v;
      bi = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi) || (ov != ov && best == best)) {
      best = ov;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi) || (ov != ov && best == best)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
  }
}

}  // namespace b2

extern "C" {

int b2_embedding(const int64_t* ids, int n, const void* table, int vocab, int dim, int dtype,
                 void* out, int out_dtype, int32_t* status, b2_stream_t stream) {
  B2_CHECK_ARG(n >= 0 && dim > 0 && vocab > 0, "b2_embedding: bad sizes n=%d dim=%d vocab=%d", n, dim, vocab);
  B2_CHECK_ARG(b2::valid_dtype(dtype) && b2::valid_dtype(out_dtype), "b2_embedding: bad dtype");
  if (n == 0) return B2_OK;
  B2_CHECK_ARG(ids && table && out, "b2_embedding: null pointer");
  b2::embedding_kernel<<<n, 256, 0, stream>>>(ids, table, vocab, dim, dtype, out, out_dtype, status);
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

int b2_rmsnorm(const void* x, int x_dtype, const void* residual, int residual_dtype, void* h_out,
               int h_dtype, const float* weight, float eps, void* y, int y_dtype, int rows, int dim,
               b2_stream_t stream) {
  B2_CHECK_ARG(rows >= 0 && dim > 0, "b2_rmsnorm: bad sizes rows=%d dim=%d", rows, dim);
  B2_CHECK_ARG(b2::valid_dtype(x_dtype) && b2::valid_dtype(y_dtype), "b2_rmsnorm: bad dtype");
  B2_CHECK_ARG(!residual || b2::valid_dtype(residual_dtype), "b2_rmsnorm: bad residual dtype");
  B2_CHECK_ARG(!h_out || b2::valid_dtype(h_dtype), "b2_rmsnorm: bad h dtype");
  B2_CHECK_ARG(dim <= 12288, "b2_rmsnorm: dim %d exceeds 12288", dim);
  if (rows == 0) return B2_OK;
  B2_CHECK_ARG(x && (y ? weight != nullptr : h_out != nullptr), "b2_rmsnorm: null pointer");
  const size_t smem = (size_t)dim * sizeof(float);
  if (smem > 48 * 1024) {
    B2_TRY_CUDA(cudaFuncSetAttribute(b2::rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
  }
  const int threads = dim >= 2048 ? 512 : (dim >= 512 ? 256 : 128);
  b2::rmsnorm_kernel<<<rows, threads, smem, stream>>>(x, x_dtype, residual, residual_dtype, h_out,
                                                     h_dtype, weight, eps, y, y_dtype, dim);
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

int b2_argmax(const float* logits, int64_t ld, int rows, int cols, int64_t* out, b2_stream_t stream) {
  B2_CHECK_ARG(rows >= 0 && cols > 0 && ld >= cols, "b2_argmax: bad sizes");
  if (rows == 0) return B2_OK;
  B2_CHECK_ARG(logits && out, "b2_argmax: null pointer");
  b2::argmax_kernel<<<rows, 512, 0, stream>>>(logits, ld, cols, out);
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

}  // extern "C"
