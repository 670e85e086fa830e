// FFMA GEMM for the float32 mode: y[m, n] = sum_k x[m, k] * w[n, k] (+ bias[n]).
//
// The reference computes every linear in float32 (engine/tensor_parallel/layers.py:83,
// :152); its parity bar for float32 is 1e-5, which tensor-core TF32 cannot meet, so
// float32 runs on the CUDA cores.  64x64 output tiles, K in steps of 16 staged
// through shared memory, 4x4 outputs per thread, float32 accumulation.
// The SwiGLU variant computes the gate and up tiles of the same columns in one CTA
// and writes silu(g) * u (engine/model/mlp.py:80-82).
#include "common.cuh"
#include "gemm.cuh"

namespace b2 {

constexpr int SBM = 64, SBN = 64, SBK = 16;

template <typename T, bool SWIGLU>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ A, int64_t lda,
                                                        const T* __restrict__ W0,
                                                        const T* __restrict__ W1, int M, int N,
                                                        int K, const float* __restrict__ bias,
                                                        void* __restrict__ Y, int64_t ldy,
                                                        int y_dtype, Scatter sc) {
  __shared__ float As[SBK][SBM + 4];
  __shared__ float Ws[SBK][SBN + 4];
  __shared__ float Us[SWIGLU ? SBK : 1][SWIGLU ? SBN + 4 : 1];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * SBM, n0 = blockIdx.x * SBN;
  float acc[4][4] = {};
  float accu[SWIGLU ? 4 : 1][SWIGLU ? 4 : 1] = {};
  for (int k0 = 0; k0 < K; k0 += SBK) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = tid + j * 256;
      const int r = e / SBK, kk = e % SBK;
      const int k = k0 + kk;
      const int m = m0 + r, n = n0 + r;
      As[kk][r] = (m < M && k < K) ? to_f32(A[(int64_t)m * lda + k]) : 0.f;
      Ws[kk][r] = (n < N && k < K) ? to_f32(W0[(int64_t)n * K + k]) : 0.f;
      if constexpr (SWIGLU) Us[kk][r] = (n < N && k < K) ? to_f32(W1[(int64_t)n * K + k]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SBK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      if constexpr (SWIGLU) {
        float u[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) u[j] = Us[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) accu[i][j] = fmaf(a[i], u[j], accu[i][j]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float v = acc[i][j];
      if constexpr (SWIGLU) {
        v = silu_f32(v) * accu[i][j];
      } else {
        if (bias) v += bias[n];
      }
      int64_t idx;
      void* base = out_base(Y, y_dtype, ldy, sc.table, sc.epoch, sc.rows_per_rank, sc.src, sc.world, m, n, &idx);
      st_dyn(base, y_dtype, idx, v);
    }
  }
}

int gemm_simt(const void* x, int64_t ldx, int M, int K, const void* w0, const void* w1, int N,
              const float* bias, void* y, int64_t ldy, int dtype, int y_dtype, cudaStream_t s,
              const Scatter* scp) {
  const Scatter sc = scp ? *scp : Scatter{nullptr, nullptr, 1, 0, 0};
  dim3 grid((N + SBN - 1) / SBN, (M + SBM - 1) / SBM);
  B2_CHECK_ARG(grid.y <= 65535, "gemm: M=%d too large", M);
  if (dtype == B2_BF16) {
    using T = __nv_bfloat16;
    if (w1)
      gemm_simt_kernel<T, true><<<grid, 256, 0, s>>>((const T*)x, ldx, (const T*)w0, (const T*)w1, M, N, K, bias, y, ldy, y_dtype, sc);
    else
      gemm_simt_kernel<T, false><<<grid, 256, 0, s>>>((const T*)x, ldx, (const T*)w0, nullptr, M, N, K, bias, y, ldy, y_dtype, sc);
  } else {
    if (w1)
      gemm_simt_kernel<float, true><<<grid, 256, 0, s>>>((const float*)x, ldx, (const float*)w0, (const float*)w1, M, N, K, bias, y, ldy, y_dtype, sc);
    else
      gemm_simt_kernel<float, false><<<grid, 256, 0, s>>>((const float*)x, ldx, (const float*)w0, nullptr, M, N, K, bias, y, ldy, y_dtype, sc);
  }
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

}  // namespace b2
