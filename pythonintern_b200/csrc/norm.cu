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
  pdl_wait();
  pdl_trigger();
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
  pdl_wait();
  pdl_trigger();
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

// Vectorised RMSNorm for rows of dim % 8 == 0 and dim <= 8 * 4 * blockDim: each thread
// keeps its (up to 4) 8-element slices of h in registers, so the row is read once.
template <typename TX>
__device__ __forceinline__ void ld8(const void* p, int dtype, size_t i, float (&v)[8]) {
  if (dtype == B2_BF16) {
    load16_f32<__nv_bfloat16>(reinterpret_cast<const __nv_bfloat16*>(p) + i, v);
  } else {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}
__device__ __forceinline__ void st8(void* p, int dtype, size_t i, const float (&v)[8]) {
  if (dtype == B2_BF16) {
    uint4 o;
    uint32_t* w = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
      w[k] = *reinterpret_cast<uint32_t*>(&h2);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p) + i) = o;
  } else {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
}

__global__ void rmsnorm_vec_kernel(const void* x, int x_dtype, const void* res, int res_dtype, void* h_out,
                                   int h_dtype, const float* __restrict__ w, float eps, void* y, int y_dtype,
                                   int dim) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const size_t base = (size_t)blockIdx.x * dim;
  const int nv = dim / 8;
  float v[4][8];
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int j = threadIdx.x + it * blockDim.x;
    if (j < nv) {
      ld8<float>(x, x_dtype, base + (size_t)j * 8, v[it]);
      if (res) {
        float r[8];
        ld8<float>(res, res_dtype, base + (size_t)j * 8, r);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[it][e] += r[e];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[it][e] * v[it][e];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)dim + eps);
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int j = threadIdx.x + it * blockDim.x;
    if (j < nv) {
      if (h_out) st8(h_out, h_dtype, base + (size_t)j * 8, v[it]);
      if (y) {
        float o[8];
        const float4 wa = *reinterpret_cast<const float4*>(w + j * 8);
        const float4 wb = *reinterpret_cast<const float4*>(w + j * 8 + 4);
        const float ww[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = v[it][e] * inv * ww[e];
        st8(y, y_dtype, base + (size_t)j * 8, o);
      }
    }
  }
}

// ---------------------------------------------------------------- argmax
// First index of the row maximum, like torch.argmax (execution_engine.py:103,133).
__global__ void argmax_kernel(const float* __restrict__ logits, int64_t ld, int cols,
                              int64_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sv[32];
  __shared__ int si[32];
  float best;
  int bi;
  block_argmax(logits + (size_t)blockIdx.x * ld, cols, sv, si, best, bi);
  if (threadIdx.x == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
}

}  // namespace b2

extern "C" {

int b2_embedding(const int64_t* ids, int n, const void* table, int vocab, int dim, int dtype,
                 void* out, int out_dtype, int32_t* status, b2_stream_t stream) {
  B2_CHECK_ARG(n >= 0 && dim > 0 && vocab > 0, "b2_embedding: bad sizes n=%d dim=%d vocab=%d", n, dim, vocab);
  B2_CHECK_ARG(b2::valid_dtype(dtype) && b2::valid_dtype(out_dtype), "b2_embedding: bad dtype");
  if (n == 0) return B2_OK;
  B2_CHECK_ARG(ids && table && out, "b2_embedding: null pointer");
  B2_TRY_CUDA(b2::launch_pdl(b2::embedding_kernel, dim3(n), dim3(256), 0, stream, ids, table, vocab, dim, dtype, out,
                              out_dtype, status));
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
  auto al16 = [](const void* q) { return q == nullptr || ((uintptr_t)q % 16) == 0; };
  if (dim % 8 == 0 && dim <= 8 * 4 * 256 && al16(x) && al16(residual) && al16(h_out) && al16(y) && al16(weight)) {
    const int nv = dim / 8;
    int threads = 32;
    while (threads < 256 && threads * 4 < nv) threads *= 2;
    while (threads < nv && threads < 256 && nv / threads > 1) threads *= 2;
    B2_TRY_CUDA(b2::launch_pdl(b2::rmsnorm_vec_kernel, dim3(rows), dim3(threads), 0, stream, x, x_dtype, residual,
                                residual_dtype, h_out, h_dtype, weight, eps, y, y_dtype, dim));
    B2_TRY_CUDA(cudaGetLastError());
    return B2_OK;
  }
  const size_t smem = (size_t)dim * sizeof(float);
  if (smem > 48 * 1024) {
    B2_TRY_CUDA(cudaFuncSetAttribute(b2::rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
  }
  const int threads = dim >= 2048 ? 512 : (dim >= 512 ? 256 : 128);
  B2_TRY_CUDA(b2::launch_pdl(b2::rmsnorm_kernel, dim3(rows), dim3(threads), smem, stream, x, x_dtype, residual,
                              residual_dtype, h_out, h_dtype, weight, eps, y, y_dtype, dim));
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

int b2_argmax(const float* logits, int64_t ld, int rows, int cols, int64_t* out, b2_stream_t stream) {
  B2_CHECK_ARG(rows >= 0 && cols > 0 && ld >= cols, "b2_argmax: bad sizes");
  if (rows == 0) return B2_OK;
  B2_CHECK_ARG(logits && out, "b2_argmax: null pointer");
  B2_TRY_CUDA(b2::launch_pdl(b2::argmax_kernel, dim3(rows), dim3(1024), 0, stream, logits, ld, cols, out));
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

}  // extern "C"
