// Shared helpers for the libb2tp kernels: status handling, dtype conversion,
// vector loads, warp reductions and bounded waits.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b2tp.h"

namespace b2 {

// Records a formatted message as the calling thread's last error and returns `status`.
int fail(int status, const char* fmt, ...);
// Number of SMs of the current device (cached per device).
int sm_count();

#define B2_TRY_CUDA(expr)                                                                  \
  do {                                                                                     \
    cudaError_t e_ = (expr);                                                               \
    if (e_ != cudaSuccess)                                                                 \
      return ::b2::fail(B2_ECUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), \
                        __FILE__, __LINE__);                                               \
  } while (0)

#define B2_CHECK_ARG(cond, ...)                           \
  do {                                                    \
    if (!(cond)) return ::b2::fail(B2_EINVAL, __VA_ARGS__); \
  } while (0)

inline bool valid_dtype(int d) { return d == B2_F32 || d == B2_BF16; }
inline size_t dtype_bytes(int d) { return d == B2_BF16 ? 2 : 4; }

// ------------------------------------------------------------------ conversions
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Runtime-typed scalar access for the small memory-bound kernels.
__device__ __forceinline__ float ld_dyn(const void* p, int dtype, size_t i) {
  return dtype == B2_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                          : reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void st_dyn(void* p, int dtype, size_t i, float v) {
  if (dtype == B2_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}

// 16-byte vector of T converted to float.
template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ void load16_f32(const T* p, float (&out)[16 / sizeof(T)]) {
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  if constexpr (sizeof(T) == 4) {
    out[0] = __uint_as_float(raw.x);
    out[1] = __uint_as_float(raw.y);
    out[2] = __uint_as_float(raw.z);
    out[3] = __uint_as_float(raw.w);
  } else {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      out[2 * i] = __uint_as_float(w[i] << 16);
      out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
}

// ------------------------------------------------------------------ reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024); `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
  if (warp == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ void raise_status(int32_t* status, int bits) {
  if (status) atomicOr(reinterpret_cast<int*>(status), bits);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// First index of the maximum of row[0, cols) over the whole CTA (blockDim a multiple of
// 32, at most 1024), like torch.argmax: ties go to the smaller index and NaN beats any
// number.  The result is valid in thread 0 (best value, index; index 0x7fffffff for an
// empty row).  sv/si: shared scratch of 32 entries each.
__device__ __forceinline__ bool argmax_better(float v, int c, float best, int bi) {
  return v > best || (v == best && c < bi) || (v != v && best == best);
}
__device__ __forceinline__ void block_argmax(const float* row, int cols, float* sv, int* si, float& best, int& bi) {
  best = -INFINITY;
  bi = 0x7fffffff;
  auto take = [&](float v, int c) {
    if (argmax_better(v, c, best, bi)) {
      best = v;
      bi = c;
    }
  };
  if ((((uintptr_t)row) & 15) == 0) {
    const int n4 = cols / 4;
    const float4* row4 = reinterpret_cast<const float4*>(row);
    int c4 = threadIdx.x;
    for (; c4 + 3 * (int)blockDim.x < n4; c4 += 4 * blockDim.x) {  // four 16-byte loads in flight
      float4 a[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = __ldg(row4 + c4 + u * blockDim.x);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = 4 * (c4 + u * blockDim.x);
        take(a[u].x, c); take(a[u].y, c + 1); take(a[u].z, c + 2); take(a[u].w, c + 3);
      }
    }
    for (; c4 < n4; c4 += blockDim.x) {
      const float4 a = __ldg(row4 + c4);
      take(a.x, 4 * c4); take(a.y, 4 * c4 + 1); take(a.z, 4 * c4 + 2); take(a.w, 4 * c4 + 3);
    }
    for (int c = 4 * n4 + threadIdx.x; c < cols; c += blockDim.x) take(row[c], c);
  } else {
    for (int c = threadIdx.x; c < cols; c += blockDim.x) take(row[c], c);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    take(ov, oi);
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
      take(ov, oi);
    }
  }
}

// Programmatic dependent launch.  Kernels of the decode step are launched with
// programmatic stream serialization (launch_pdl), so the next kernel in the stream can be
// scheduled while the current one drains.  Every such kernel calls pdl_wait() before it
// touches global memory that an earlier kernel writes or reads (griddepcontrol.wait
// returns once the preceding grid has completed and its writes are visible; it returns
// at once when there is no programmatic predecessor), then pdl_trigger() to let its own
// successor be scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace b2
