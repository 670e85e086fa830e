// Tensor-parallel all-reduce over NVLink peer memory.
//
// Replaces the reference's gRPC all-reduce (engine/tensor_parallel/comm.py:72-154,
// buffer_codec.py:27-69, worker_node.py:107-125), in which every rank serialises its
// partial tensor, sends it to every peer and sums what arrives.  Here every rank owns one
// device allocation, exported once through a CUDA IPC handle:
//
//     [ data[0] | data[1] | recv[3] | xn[3] | flags[8][kMaxCtas] | ctrl | scatter table | amx[3][8][4096] ]
//
// * One-shot module API (b2_allreduce_sum / b2_allreduce_rmsnorm): the partial goes into
//   data[parity]; each CTA raises flag[rank][cta] = epoch on every peer (st.release.sys),
//   waits for the peers' flags with a %globaltimer bound (ld.acquire.sys), then loads every
//   rank's partial over NVLink and sums in rank order 0..world-1 (bit-identical on all
//   ranks); the fused variant adds the float32 residual and applies the next RMSNorm.
//   Two data buffers alternate by call parity.
// * Decode path (b2_row_parallel_linear + b2_allreduce_rmsnorm_sharded), flag free: the
//   row-parallel GEMM's epilogue stores each output row into recv[b] of the rank that
//   owns the row; the owner sums the sources in rank order, adds its float32 residual
//   slice, normalises, and stores the row into xn[b] of every rank; every rank copies
//   its xn[b] out.  Idle slots hold a sentinel (all-ones bytes, a NaN payload that
//   arithmetic never produces), so the arrival of every element is its own signal; the
//   slots rotate over three values of a device-side epoch (b = epoch % 3) and a slot is
//   refilled with the sentinel one call after it was consumed, which leaves a full call
//   of slack before any rank can write it again.
// * Greedy sampling over a vocab-parallel lm_head (b2_argmax_allgather): each rank stores
//   its (max, index) per row into amx[b] of every rank, sentinel-checked the same way.
// Epochs advance on the device (last CTA of a call), so CUDA-graph replays need no host
// bookkeeping; every wait is bounded and raises B2_DEV_PEER_TIMEOUT.
#include <cstring>
#include <new>

#include "common.cuh"
#include "gemm.cuh"

namespace b2 {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 128;

constexpr int kSlots = 3;  // rotating receive slots of the flag-free fused path
constexpr int kMaxArgRows = 4096;  // rows of one vocab-parallel argmax exchange

struct CommView {
  void* data[2][kMaxRanks];        // every rank's one-shot data buffers (own included)
  void* xn[kSlots][kMaxRanks];     // every rank's all-gather slots of normalised rows
  void* recv_own[kSlots];          // this rank's reduce-scatter receive slots
  uint32_t* flags[kMaxRanks];      // every rank's flag array [kMaxRanks][kMaxCtas]
  char* amx[kMaxRanks];             // every rank's argmax exchange slots [kSlots][kMaxRanks][kMaxArgRows]
  uint32_t* ctrl;                  // own control words (epochs, done counters, slot extents)
  size_t slot_bytes;
  int rank, world;
};

}  // namespace b2

struct b2_comm {
  int rank, world, device;
  size_t max_bytes, data_bytes;
  size_t off_data[2], off_recv[b2::kSlots], off_xn[b2::kSlots], off_flags, off_ctrl, off_table, off_amx, total;
  unsigned long long* scatter_table;  // device: [kSlots][kMaxRanks] every rank's receive slot addresses
  char* base;                       // own allocation
  char* peer_base[b2::kMaxRanks];   // mapped peers (own base at [rank])
  cudaIpcMemHandle_t handle;
  bool opened;
  bool local_peers;  // peers wired in-process by b2_comm_open_local (no IPC mappings to close)
};

namespace b2 {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Steps 1-2 of the flag protocol.  Returns false (and raises the status bit) on timeout.
__device__ bool comm_barrier(const CommView& v, uint32_t epoch, int64_t timeout_ns, int32_t* status) {
  __shared__ int s_ok;
  const int cta = blockIdx.x;
  const int pofs = 0;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < v.world) {
    __threadfence_system();
    st_release_sys(v.flags[threadIdx.x] + pofs + v.rank * kMaxCtas + cta, epoch);
  }
  if (threadIdx.x < v.world) {
    const uint32_t* f = v.flags[v.rank] + pofs + threadIdx.x * kMaxCtas + cta;
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
      if ((++it & 255) == 0 && (int64_t)(globaltimer_ns() - t0) > timeout_ns) {
        raise_status(status, B2_DEV_PEER_TIMEOUT);
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  return s_ok != 0;
}

// Last CTA to finish advances the epoch for the next call.
__device__ void comm_finish(const CommView& v) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(v.ctrl + 1, 1u);
    if (prev == gridDim.x - 1) {
      v.ctrl[1] = 0;
      v.ctrl[0] = v.ctrl[0] + 1;
      __threadfence();
    }
  }
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&o)[8]);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&o)[8]) {
  const uint4 raw = __ldcv(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = __uint_as_float(w[i] << 16);
    o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&o)[8]) {
  const float4 a = __ldcv(reinterpret_cast<const float4*>(p));
  const float4 b = __ldcv(reinterpret_cast<const float4*>(p) + 1);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
  o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}

template <typename T>
__device__ __forceinline__ void store8(T* dst, const float (&v)[8]);
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* dst, const float (&v)[8]) {
  uint4 o;
  uint32_t* w = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
    w[k] = *reinterpret_cast<uint32_t*>(&h2);
  }
  *reinterpret_cast<uint4*>(dst) = o;
}
template <>
__device__ __forceinline__ void store8<float>(float* dst, const float (&v)[8]) {
  reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// out[i] = sum_r data_r[parity][i], 8 elements per thread step.
template <typename T>
__global__ void allreduce_sum_kernel(CommView v, int parity, size_t n8, T* __restrict__ out,
                                     int64_t timeout_ns, int32_t* status) {
  const uint32_t epoch = v.ctrl[0] + 1;
  if (comm_barrier(v, epoch, timeout_ns, status)) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int r = 0; r < v.world; ++r) {
        float x[8];
        load8<T>(reinterpret_cast<const T*>(v.data[parity][r]) + i * 8, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += x[e];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) out[i * 8 + e] = from_f32<T>(acc[e]);
    }
  }
  comm_finish(v);
}

// h = residual + sum_r data_r[parity] (row-major [rows, dim]); y = rmsnorm(h) * w.
template <typename T>
__global__ void allreduce_rmsnorm_kernel(CommView v, int parity, int rows, int dim,
                                         const float* residual, float* h_out,
                                         const float* __restrict__ w, float eps, void* y,
                                         int y_dtype, int64_t timeout_ns, int32_t* status) {
  extern __shared__ float srow[];
  __shared__ float red[32];
  const uint32_t epoch = v.ctrl[0] + 1;
  if (comm_barrier(v, epoch, timeout_ns, status)) {
    const int nv = dim / 8;
    for (int row = blockIdx.x; row < rows; row += gridDim.x) {
      const size_t base = (size_t)row * dim;
      float ss = 0.f;
      for (int j = threadIdx.x; j < nv; j += blockDim.x) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int r = 0; r < v.world; ++r) {
          float x[8];
          load8<T>(reinterpret_cast<const T*>(v.data[parity][r]) + base + j * 8, x);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += x[e];
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float h = (residual ? residual[base + j * 8 + e] : 0.f) + acc[e];
          srow[j * 8 + e] = h;
          ss += h * h;
        }
      }
      ss = block_sum(ss, red);
      const float inv = rsqrtf(ss / (float)dim + eps);
      for (int c = threadIdx.x; c < dim; c += blockDim.x) {
        const float h = srow[c];
        if (h_out) h_out[base + c] = h;
        st_dyn(y, y_dtype, base + c, h * inv * w[c]);
      }
      __syncthreads();
    }
  }
  comm_finish(v);
}

// Sentinel helpers: a slot element still equal to the all-ones pattern has not arrived.
__device__ __forceinline__ uint4 ld_volatile16(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
template <typename T>
__device__ __forceinline__ bool has_sentinel(const uint4& v) {
  if (sizeof(T) == 4) return v.x == 0xffffffffu || v.y == 0xffffffffu || v.z == 0xffffffffu || v.w == 0xffffffffu;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if ((w[k] & 0xffffu) == 0xffffu || (w[k] >> 16) == 0xffffu) return true;
  return false;
}
// Waits (bounded by deadline) until the 16 bytes at p hold no sentinel element.
template <typename T>
__device__ __forceinline__ uint4 wait16(const void* p, uint64_t deadline, bool* ok) {
  uint4 v = ld_volatile16(p);
  uint32_t it = 0;
  while (has_sentinel<T>(v)) {
    if ((++it & 63) == 0 && globaltimer_ns() > deadline) {
      *ok = false;
      return v;
    }
    v = ld_volatile16(p);
  }
  return v;
}
__device__ __forceinline__ void unpack8(const uint4& raw, float (&o)[8], bool bf16) {
  if (bf16) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[2 * i] = __uint_as_float(w[i] << 16);
      o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
}

// Second half of the fused row-parallel all-reduce (flag free).  Slot b = epoch % 3.
//  A. CTA c owns rows rank*R + c, + gridDim.x, ... (a prefill can give a rank more rows
//     than the grid has CTAs): per row it waits for each source's partial in its receive
//     slot b, sums them in rank order, adds the float32 residual slice, normalises, and
//     stores the normalised row into slot b of EVERY rank's all-gather buffer.  Part A
//     waits only on the peers' GEMMs, never on another CTA of this grid, and every CTA
//     finishes its part A rows before part C, so the grid-stride loop cannot deadlock.
//  B. every CTA refills its share of the slots used by the previous call ((b + 2) % 3)
//     with the sentinel.
//  C. every CTA waits for its share of rows of its own all-gather slot b and copies them
//     to y (the caller's [rows, dim] output).
template <typename T, bool MULTI>
__global__ void __launch_bounds__(512) allreduce_rmsnorm_sharded_kernel(CommView v, int rows, int R, int dim, float* h_slice,
                                                 const float* __restrict__ w, float eps, T* __restrict__ y,
                                                 int64_t timeout_ns, int32_t* status) {
  // No griddepcontrol.wait: everything this kernel reads from the preceding GEMM arrives
  // through the sentinel-checked receive slot, and the rest (epoch, extents, residual
  // slice) was last written by the previous call of this kernel, which the GEMM itself
  // waited for.  So its CTAs start polling as soon as the GEMM's CTAs free their SMs.
  pdl_trigger();
  __shared__ float red[32];
  __shared__ int s_ok;
  const uint32_t epoch = v.ctrl[0];
  const int b = (int)(epoch % kSlots);
  const int prev = (b + kSlots - 1) % kSlots;
  const uint64_t deadline = globaltimer_ns() + (uint64_t)timeout_ns;
  const int nv = dim / 8;
  constexpr bool BF = sizeof(T) == 2;
  bool ok = true;
  if (threadIdx.x == 0) s_ok = 1;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    v.ctrl[2 + b] = (uint32_t)(((size_t)v.world * R * dim * sizeof(T)) / 16);
    v.ctrl[5 + b] = (uint32_t)(((size_t)rows * dim * sizeof(T)) / 16);
  }
  __syncthreads();

  // A. reduce the owned rows (MULTI: more owned rows than CTAs, each CTA loops)
  auto reduce_row = [&](const int rr, const int row) {
    const T* recv = reinterpret_cast<const T*>(v.recv_own[b]);
    float hv[4][8];
    float4 wv[4][2];
    float ss = 0.f;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int j = threadIdx.x + it * blockDim.x;
      if (j >= nv) continue;
      // residual and norm weight are requested first; they do not depend on the partials
      float* hp = h_slice + (size_t)rr * dim + j * 8;
      const float4 h0 = *reinterpret_cast<const float4*>(hp);
      const float4 h1 = *reinterpret_cast<const float4*>(hp + 4);
      wv[it][0] = __ldg(reinterpret_cast<const float4*>(w + j * 8));
      wv[it][1] = __ldg(reinterpret_cast<const float4*>(w + j * 8) + 1);
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      // every source's vector is loaded before any is checked, so the common case costs
      // one round of independent loads; only vectors that have not arrived are polled again
      constexpr int NV16 = BF ? 1 : 2;  // 16-byte loads per 8 elements
      uint4 raw[NV16 * kMaxRanks];
#pragma unroll
      for (int src = 0; src < kMaxRanks; ++src) {
        if (src >= v.world) break;
        const T* ptr = recv + ((size_t)src * R + rr) * dim + j * 8;
#pragma unroll
        for (int h = 0; h < NV16; ++h) raw[src * NV16 + h] = ld_volatile16(ptr + h * (8 / NV16));
      }
#pragma unroll
      for (int src = 0; src < kMaxRanks; ++src) {
        if (src >= v.world) break;
        const T* ptr = recv + ((size_t)src * R + rr) * dim + j * 8;
#pragma unroll
        for (int h = 0; h < NV16; ++h)
          if (has_sentinel<T>(raw[src * NV16 + h])) raw[src * NV16 + h] = wait16<T>(ptr + h * (8 / NV16), deadline, &ok);
        float x[8];
        if (BF) {
          unpack8(raw[src * NV16], x, true);
        } else {
          const uint4 r0 = raw[src * NV16], r1 = raw[src * NV16 + NV16 - 1];
          x[0] = __uint_as_float(r0.x); x[1] = __uint_as_float(r0.y); x[2] = __uint_as_float(r0.z); x[3] = __uint_as_float(r0.w);
          x[4] = __uint_as_float(r1.x); x[5] = __uint_as_float(r1.y); x[6] = __uint_as_float(r1.z); x[7] = __uint_as_float(r1.w);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += x[e];
      }
      const float hr[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        hv[it][e] = hr[e] + acc[e];
        ss += hv[it][e] * hv[it][e];
      }
      *reinterpret_cast<float4*>(hp) = make_float4(hv[it][0], hv[it][1], hv[it][2], hv[it][3]);
      *reinterpret_cast<float4*>(hp + 4) = make_float4(hv[it][4], hv[it][5], hv[it][6], hv[it][7]);
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)dim + eps);
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int j = threadIdx.x + it * blockDim.x;
      if (j >= nv) continue;
      const float wr[8] = {wv[it][0].x, wv[it][0].y, wv[it][0].z, wv[it][0].w,
                           wv[it][1].x, wv[it][1].y, wv[it][1].z, wv[it][1].w};
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = hv[it][e] * inv * wr[e];
      for (int q = 0; q < v.world; ++q)
        store8<T>(reinterpret_cast<T*>(v.xn[b][q]) + (size_t)row * dim + j * 8, o);
    }
  };
  if constexpr (MULTI) {
    for (int rr = blockIdx.x; rr < R; rr += gridDim.x) {
      const int row = v.rank * R + rr;
      if (row >= rows) break;
      reduce_row(rr, row);
    }
  } else {
    const int row = v.rank * R + blockIdx.x;
    if (blockIdx.x < R && row < rows) reduce_row(blockIdx.x, row);
  }

  // B. re-arm the previous call's slots (receive slot and own all-gather slot) over the
  //    extents that call used, which ctrl[2 + slot] / ctrl[5 + slot] record in 16-byte units.
  {
    const size_t recv_n16 = v.ctrl[2 + prev];
    const size_t xn_n16 = v.ctrl[5 + prev];
    uint4* r16 = reinterpret_cast<uint4*>(v.recv_own[prev]);
    uint4* x16 = reinterpret_cast<uint4*>(v.xn[prev][v.rank]);
    const uint4 ones = make_uint4(0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < recv_n16; i += (size_t)gridDim.x * blockDim.x)
      r16[i] = ones;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < xn_n16; i += (size_t)gridDim.x * blockDim.x)
      x16[i] = ones;
  }

  // C. wait for the all-gathered rows and copy them out, four independent loads per round
  {
    const uint4* xs = reinterpret_cast<const uint4*>(v.xn[b][v.rank]);
    uint4* yd = reinterpret_cast<uint4*>(y);
    const size_t n16 = ((size_t)rows * dim * sizeof(T)) / 16;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n16; i0 += 4 * stride) {
      uint4 r[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u * stride < n16) r[u] = ld_volatile16(xs + i0 + u * stride);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const size_t i = i0 + u * stride;
        if (i >= n16) break;
        if (has_sentinel<T>(r[u])) r[u] = wait16<T>(xs + i, deadline, &ok);
        yd[i] = r[u];
      }
    }
  }
  if (!ok) {
    raise_status(status, B2_DEV_PEER_TIMEOUT);
    s_ok = 0;
  }
  comm_finish(v);
}

// Greedy token over a vocab-parallel lm_head (the replicated-logits argmax of
// execution_engine.py:103,133).  CTA per row: the block argmax over this rank's vocab
// slice, then thread 0 stores (value bits << 32 | global index) into slot b of every
// rank's exchange buffer and waits (sentinel polling, bounded) for the world's entries of
// its row, taking the best in rank order: rank order is vocab order, so a tie keeps the
// smaller index and the first NaN wins, exactly as an argmax over the full row.  The slot
// of the previous call is re-armed; the last CTA advances the exchange epoch (ctrl[8]).
__global__ void __launch_bounds__(1024) argmax_allgather_kernel(CommView v, const float* __restrict__ logits,
                                                                int64_t ld, int rows, int cols, int64_t vocab_offset,
                                                                int64_t* __restrict__ out, int64_t timeout_ns,
                                                                int32_t* status) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sv[32];
  __shared__ int si[32];
  const uint32_t epoch = v.ctrl[8];
  const int b = (int)(epoch % kSlots);
  const int prev = (b + kSlots - 1) % kSlots;
  if (blockIdx.x == 0 && threadIdx.x == 0) v.ctrl[10 + b] = (uint32_t)rows;
  float best;
  int bi;
  block_argmax(logits + (size_t)blockIdx.x * ld, cols, sv, si, best, bi);
  if (threadIdx.x == 0) {
    const uint32_t gidx = (uint32_t)(vocab_offset + (bi == 0x7fffffff ? 0 : bi));
    const unsigned long long packed = ((unsigned long long)__float_as_uint(best) << 32) | gidx;
    for (int q = 0; q < v.world; ++q) {
      unsigned long long* dst = reinterpret_cast<unsigned long long*>(v.amx[q]) +
                                ((size_t)(b * kMaxRanks + v.rank) * kMaxArgRows + blockIdx.x);
      *reinterpret_cast<volatile unsigned long long*>(dst) = packed;
    }
    const uint64_t deadline = globaltimer_ns() + (uint64_t)timeout_ns;
    const unsigned long long* own = reinterpret_cast<const unsigned long long*>(v.amx[v.rank]);
    float bv = 0.f;
    uint32_t bidx = 0;
    bool ok = true;
    for (int src = 0; src < v.world && ok; ++src) {
      const volatile unsigned long long* p = own + ((size_t)(b * kMaxRanks + src) * kMaxArgRows + blockIdx.x);
      unsigned long long x = *p;
      uint32_t it = 0;
      while (x == ~0ull) {
        if ((++it & 63) == 0 && globaltimer_ns() > deadline) {
          ok = false;
          break;
        }
        x = *p;
      }
      if (!ok) break;
      const float xv = __uint_as_float((uint32_t)(x >> 32));
      if (src == 0 || xv > bv || (xv != xv && bv == bv)) {
        bv = xv;
        bidx = (uint32_t)x;
      }
    }
    if (!ok) raise_status(status, B2_DEV_PEER_TIMEOUT);
    out[blockIdx.x] = (int64_t)bidx;
  }
  // Re-arm this rank's slot of the previous call, over the rows that call used.
  const int prow = (int)v.ctrl[10 + prev];
  unsigned long long* own_prev = reinterpret_cast<unsigned long long*>(v.amx[v.rank]) + (size_t)prev * kMaxRanks * kMaxArgRows;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < v.world * prow; i += gridDim.x * blockDim.x)
    own_prev[(size_t)(i / prow) * kMaxArgRows + (i % prow)] = ~0ull;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t d = atomicAdd(v.ctrl + 9, 1u);
    if (d == gridDim.x - 1) {
      v.ctrl[9] = 0;
      v.ctrl[8] = epoch + 1;
      __threadfence();
    }
  }
}

static CommView make_view(const b2_comm* c) {
  CommView v{};
  v.rank = c->rank;
  v.world = c->world;
  for (int r = 0; r < c->world; ++r) {
    v.data[0][r] = c->peer_base[r] + c->off_data[0];
    v.data[1][r] = c->peer_base[r] + c->off_data[1];
    for (int k = 0; k < kSlots; ++k) v.xn[k][r] = c->peer_base[r] + c->off_xn[k];
    v.flags[r] = reinterpret_cast<uint32_t*>(c->peer_base[r] + c->off_flags);
    v.amx[r] = c->peer_base[r] + c->off_amx;
  }
  for (int k = 0; k < kSlots; ++k) v.recv_own[k] = c->base + c->off_recv[k];
  v.slot_bytes = c->data_bytes;
  v.ctrl = reinterpret_cast<uint32_t*>(c->base + c->off_ctrl);
  return v;
}

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Fills the device table of every rank's data-buffer address (as seen from this rank).
static int fill_scatter_table(b2_comm* c) {
  unsigned long long t[kSlots * kMaxRanks] = {0};
  for (int k = 0; k < kSlots; ++k)
    for (int r = 0; r < c->world; ++r)
      t[k * kMaxRanks + r] = (unsigned long long)(uintptr_t)(c->peer_base[r] + c->off_recv[k]);
  int dev = 0;
  B2_TRY_CUDA(cudaGetDevice(&dev));
  B2_TRY_CUDA(cudaSetDevice(c->device));
  cudaError_t e = cudaMemcpy(c->scatter_table, t, sizeof(t), cudaMemcpyHostToDevice);
  cudaSetDevice(dev);
  if (e != cudaSuccess) return fail(B2_ECUDA, "scatter table upload: %s", cudaGetErrorString(e));
  return B2_OK;
}

}  // namespace b2

extern "C" {

size_t b2_comm_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int b2_comm_create(int rank, int world_size, size_t max_bytes, b2_comm** out) {
  B2_CHECK_ARG(out, "b2_comm_create: null out");
  B2_CHECK_ARG(world_size >= 1 && world_size <= b2::kMaxRanks, "b2_comm_create: world_size %d not in [1, 8]", world_size);
  B2_CHECK_ARG(rank >= 0 && rank < world_size, "b2_comm_create: rank %d out of range", rank);
  B2_CHECK_ARG(max_bytes > 0, "b2_comm_create: max_bytes must be > 0");
  b2_comm* c = new (std::nothrow) b2_comm();
  if (!c) return b2::fail(B2_EINVAL, "b2_comm_create: out of host memory");
  c->rank = rank;
  c->world = world_size;
  B2_TRY_CUDA(cudaGetDevice(&c->device));
  c->max_bytes = max_bytes;
  c->data_bytes = b2::align_up(max_bytes, 4096);
  c->off_data[0] = 0;
  c->off_data[1] = c->data_bytes;
  for (int k = 0; k < b2::kSlots; ++k) {
    c->off_recv[k] = (2 + k) * c->data_bytes;
    c->off_xn[k] = (2 + b2::kSlots + k) * c->data_bytes;
  }
  c->off_flags = (2 + 2 * b2::kSlots) * c->data_bytes;
  c->off_ctrl = c->off_flags + b2::align_up((size_t)b2::kMaxRanks * b2::kMaxCtas * sizeof(uint32_t), 256);
  c->off_table = c->off_ctrl + 256;
  c->off_amx = c->off_table + 256;
  c->total = c->off_amx + (size_t)b2::kSlots * b2::kMaxRanks * b2::kMaxArgRows * sizeof(uint64_t);
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&c->base), c->total);
  if (e != cudaSuccess) {
    delete c;
    return b2::fail(B2_ECUDA, "b2_comm_create: cudaMalloc(%zu): %s", (size_t)0, cudaGetErrorString(e));
  }
  e = cudaMemset(c->base + c->off_flags, 0, c->off_amx - c->off_flags);
  if (e == cudaSuccess) e = cudaMemset(c->base + c->off_amx, 0xff, c->total - c->off_amx);
  if (e == cudaSuccess) e = cudaMemset(c->base, 0, 2 * c->data_bytes);
  // idle receive and all-gather slots hold the sentinel
  if (e == cudaSuccess) e = cudaMemset(c->base + c->off_recv[0], 0xff, 2 * b2::kSlots * c->data_bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&c->handle, c->base);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(c->base);
    delete c;
    return b2::fail(B2_ECUDA, "b2_comm_create: %s", cudaGetErrorString(e));
  }
  for (int r = 0; r < b2::kMaxRanks; ++r) c->peer_base[r] = nullptr;
  c->peer_base[rank] = c->base;
  c->scatter_table = reinterpret_cast<unsigned long long*>(c->base + c->off_table);
  c->opened = world_size == 1;
  c->local_peers = false;
  if (world_size == 1) {
    const int rc = b2::fill_scatter_table(c);
    if (rc) {
      cudaFree(c->base);
      delete c;
      return rc;
    }
  }
  *out = c;
  return B2_OK;
}

int b2_comm_export_handle(b2_comm* comm, void* handle, size_t len) {
  B2_CHECK_ARG(comm && handle && len >= sizeof(cudaIpcMemHandle_t), "b2_comm_export_handle: bad arguments");
  memcpy(handle, &comm->handle, sizeof(cudaIpcMemHandle_t));
  return B2_OK;
}

int b2_comm_open_peers(b2_comm* comm, const void* all_handles, size_t len) {
  B2_CHECK_ARG(comm && all_handles, "b2_comm_open_peers: null argument");
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  B2_CHECK_ARG(len >= hb * comm->world, "b2_comm_open_peers: %zu bytes given, %zu needed", len, hb * comm->world);
  B2_CHECK_ARG(!comm->opened || comm->world == 1, "b2_comm_open_peers: already opened");
  const char* h = static_cast<const char*>(all_handles);
  for (int r = 0; r < comm->world; ++r) {
    if (r == comm->rank) continue;
    cudaIpcMemHandle_t ph;
    memcpy(&ph, h + r * hb, hb);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, ph, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != comm->rank && comm->peer_base[q]) {
          cudaIpcCloseMemHandle(comm->peer_base[q]);
          comm->peer_base[q] = nullptr;
        }
      return b2::fail(B2_ECUDA, "b2_comm_open_peers: rank %d handle: %s", r, cudaGetErrorString(e));
    }
    comm->peer_base[r] = static_cast<char*>(p);
  }
  comm->opened = true;
  return b2::fill_scatter_table(comm);
}

int b2_comm_open_local(b2_comm* const* comms, int n) {
  B2_CHECK_ARG(comms && n >= 1 && n <= b2::kMaxRanks, "b2_comm_open_local: bad arguments");
  for (int i = 0; i < n; ++i) {
    B2_CHECK_ARG(comms[i] && comms[i]->world == n && comms[i]->rank == i,
                 "b2_comm_open_local: comms[%d] must be rank %d of a world of %d", i, i, n);
    for (int j = 0; j < i; ++j)
      B2_CHECK_ARG(comms[i]->device != comms[j]->device,
                   "b2_comm_open_local: ranks %d and %d share device %d (one GPU per rank)", j, i, comms[i]->device);
  }
  int dev = 0;
  B2_TRY_CUDA(cudaGetDevice(&dev));
  for (int i = 0; i < n; ++i) {
    B2_TRY_CUDA(cudaSetDevice(comms[i]->device));
    for (int j = 0; j < n; ++j) {
      if (j == i) continue;
      int can = 0;
      B2_TRY_CUDA(cudaDeviceCanAccessPeer(&can, comms[i]->device, comms[j]->device));
      if (!can) {
        cudaSetDevice(dev);
        return b2::fail(B2_ENOTSUP, "b2_comm_open_local: device %d cannot access device %d", comms[i]->device, comms[j]->device);
      }
      cudaError_t e = cudaDeviceEnablePeerAccess(comms[j]->device, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
      } else if (e != cudaSuccess) {
        cudaSetDevice(dev);
        return b2::fail(B2_ECUDA, "b2_comm_open_local: enable peer access %d->%d: %s", comms[i]->device, comms[j]->device, cudaGetErrorString(e));
      }
    }
  }
  B2_TRY_CUDA(cudaSetDevice(dev));
  for (int i = 0; i < n; ++i) {
    for (int j = 0; j < n; ++j) comms[i]->peer_base[j] = comms[j]->base;
    comms[i]->opened = true;
    comms[i]->local_peers = true;
    const int rc = b2::fill_scatter_table(comms[i]);
    if (rc) return rc;
  }
  return B2_OK;
}

int b2_comm_buffer(b2_comm* comm, int parity, void** ptr) {
  B2_CHECK_ARG(comm && ptr && (parity == 0 || parity == 1), "b2_comm_buffer: bad arguments");
  *ptr = comm->base + comm->off_data[parity];
  return B2_OK;
}

int b2_comm_destroy(b2_comm* comm) {
  if (!comm) return B2_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaSetDevice(comm->device);
  cudaDeviceSynchronize();
  if (!comm->local_peers)
    for (int r = 0; r < comm->world; ++r)
      if (r != comm->rank && comm->peer_base[r]) cudaIpcCloseMemHandle(comm->peer_base[r]);
  cudaFree(comm->base);
  cudaSetDevice(dev);
  delete comm;
  return B2_OK;
}

int b2_allreduce_sum(b2_comm* comm, int parity, size_t count, int dtype, void* out,
                     int64_t timeout_ns, int32_t* status, b2_stream_t stream) {
  B2_CHECK_ARG(comm && comm->opened, "b2_allreduce_sum: communicator not opened");
  B2_CHECK_ARG(parity == 0 || parity == 1, "b2_allreduce_sum: parity must be 0 or 1");
  B2_CHECK_ARG(b2::valid_dtype(dtype), "b2_allreduce_sum: bad dtype");
  B2_CHECK_ARG(count % 8 == 0, "b2_allreduce_sum: count must be a multiple of 8");
  B2_CHECK_ARG(count * b2::dtype_bytes(dtype) <= comm->max_bytes, "b2_allreduce_sum: %zu elements exceed the buffer", count);
  B2_CHECK_ARG(out && ((uintptr_t)out % 16) == 0, "b2_allreduce_sum: out must be 16-byte aligned");
  if (count == 0) return B2_OK;
  const b2::CommView v = b2::make_view(comm);
  const size_t n8 = count / 8;
  int grid = (int)((n8 + 255) / 256);
  if (grid > b2::kMaxCtas) grid = b2::kMaxCtas;
  if (grid < 1) grid = 1;
  if (dtype == B2_BF16)
    b2::allreduce_sum_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(v, parity, n8, (__nv_bfloat16*)out, timeout_ns, status);
  else
    b2::allreduce_sum_kernel<float><<<grid, 256, 0, stream>>>(v, parity, n8, (float*)out, timeout_ns, status);
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

int b2_allreduce_rmsnorm(b2_comm* comm, int parity, int rows, int dim, int dtype,
                         const float* residual, float* h_out, const float* norm_w, float eps,
                         void* y, int y_dtype, int64_t timeout_ns, int32_t* status,
                         b2_stream_t stream) {
  B2_CHECK_ARG(comm && comm->opened, "b2_allreduce_rmsnorm: communicator not opened");
  B2_CHECK_ARG(parity == 0 || parity == 1, "b2_allreduce_rmsnorm: parity must be 0 or 1");
  B2_CHECK_ARG(b2::valid_dtype(dtype) && b2::valid_dtype(y_dtype), "b2_allreduce_rmsnorm: bad dtype");
  B2_CHECK_ARG(rows >= 0 && dim > 0 && dim % 8 == 0 && dim <= 12288, "b2_allreduce_rmsnorm: bad dim %d", dim);
  B2_CHECK_ARG((size_t)rows * dim * b2::dtype_bytes(dtype) <= comm->max_bytes, "b2_allreduce_rmsnorm: payload exceeds the buffer");
  if (rows == 0) return B2_OK;
  B2_CHECK_ARG(norm_w && y, "b2_allreduce_rmsnorm: null pointer");
  const b2::CommView v = b2::make_view(comm);
  const int grid = rows < b2::kMaxCtas ? rows : b2::kMaxCtas;
  const int threads = dim >= 4096 ? 512 : 256;
  const size_t smem = (size_t)dim * sizeof(float);
  if (dtype == B2_BF16) {
    if (smem > 48 * 1024)
      B2_TRY_CUDA(cudaFuncSetAttribute(b2::allreduce_rmsnorm_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    b2::allreduce_rmsnorm_kernel<__nv_bfloat16><<<grid, threads, smem, stream>>>(
        v, parity, rows, dim, residual, h_out, norm_w, eps, y, y_dtype, timeout_ns, status);
  } else {
    if (smem > 48 * 1024)
      B2_TRY_CUDA(cudaFuncSetAttribute(b2::allreduce_rmsnorm_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    b2::allreduce_rmsnorm_kernel<float><<<grid, threads, smem, stream>>>(
        v, parity, rows, dim, residual, h_out, norm_w, eps, y, y_dtype, timeout_ns, status);
  }
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

int b2_row_parallel_linear(b2_comm* comm, const void* x, int64_t ldx, int M, int K, const void* w, int N,
                           int dtype, void* workspace, size_t workspace_bytes, int32_t* status,
                           b2_stream_t stream) {
  B2_CHECK_ARG(comm && comm->opened, "b2_row_parallel_linear: communicator not opened");
  B2_CHECK_ARG(b2::valid_dtype(dtype), "b2_row_parallel_linear: bad dtype");
  B2_CHECK_ARG(M >= 0 && K > 0 && N > 0 && ldx >= K, "b2_row_parallel_linear: bad sizes");
  if (M == 0) return B2_OK;
  B2_CHECK_ARG(x && w, "b2_row_parallel_linear: null pointer");
  const int R = (M + comm->world - 1) / comm->world;
  B2_CHECK_ARG((size_t)comm->world * R * N * b2::dtype_bytes(dtype) <= comm->max_bytes,
               "b2_row_parallel_linear: %d x %d partial exceeds the communicator buffer", M, N);
  b2::Scatter sc{comm->scatter_table, reinterpret_cast<const unsigned int*>(comm->base + comm->off_ctrl), R,
                 comm->rank, comm->world};
  if (dtype == B2_F32) return b2::gemm_simt(x, ldx, M, K, w, nullptr, N, nullptr, nullptr, N, dtype, dtype, stream, &sc);
  b2::GemmSeg seg{w, N, 0};
  return b2::gemm_tc(x, ldx, M, K, &seg, 1, b2::kEpiStore, nullptr, nullptr, N, dtype, workspace, workspace_bytes,
                     status, stream, &sc);
}

int b2_argmax_allgather(b2_comm* comm, const float* logits, int64_t ld, int rows, int cols, int64_t vocab_offset,
                        int64_t* out, int64_t timeout_ns, int32_t* status, b2_stream_t stream) {
  B2_CHECK_ARG(comm && comm->opened, "b2_argmax_allgather: communicator not opened");
  B2_CHECK_ARG(rows >= 0 && rows <= b2::kMaxArgRows, "b2_argmax_allgather: %d rows (at most %d)", rows, b2::kMaxArgRows);
  B2_CHECK_ARG(cols > 0 && ld >= cols && vocab_offset >= 0 && vocab_offset + cols < (int64_t)0x7fffffff,
               "b2_argmax_allgather: bad sizes cols=%d ld=%lld offset=%lld", cols, (long long)ld, (long long)vocab_offset);
  if (rows == 0) return B2_OK;
  B2_CHECK_ARG(logits && out, "b2_argmax_allgather: null pointer");
  const b2::CommView v = b2::make_view(comm);
  B2_TRY_CUDA(b2::launch_pdl(b2::argmax_allgather_kernel, dim3(rows), dim3(1024), 0, stream, v, logits, ld, rows,
                             cols, vocab_offset, out, timeout_ns, status));
  return B2_OK;
}

int b2_allreduce_rmsnorm_sharded(b2_comm* comm, int rows, int dim, int dtype, float* h_slice, const float* norm_w,
                                 float eps, void* y, int64_t timeout_ns, int32_t* status, b2_stream_t stream) {
  B2_CHECK_ARG(comm && comm->opened, "b2_allreduce_rmsnorm_sharded: communicator not opened");
  B2_CHECK_ARG(b2::valid_dtype(dtype), "b2_allreduce_rmsnorm_sharded: bad dtype");
  B2_CHECK_ARG(rows >= 0 && dim > 0 && dim % 8 == 0 && dim <= 8 * 4 * 512,
               "b2_allreduce_rmsnorm_sharded: bad dim %d", dim);
  if (rows == 0) return B2_OK;
  const int R = (rows + comm->world - 1) / comm->world;
  B2_CHECK_ARG((size_t)comm->world * R * dim * b2::dtype_bytes(dtype) <= comm->max_bytes,
               "b2_allreduce_rmsnorm_sharded: payload exceeds the buffer");
  B2_CHECK_ARG(norm_w && y && (h_slice || comm->rank * R >= rows), "b2_allreduce_rmsnorm_sharded: null pointer");
  B2_CHECK_ARG(((uintptr_t)h_slice % 16) == 0 && ((uintptr_t)norm_w % 16) == 0 && ((uintptr_t)y % 16) == 0,
               "b2_allreduce_rmsnorm_sharded: h_slice, norm_w and y must be 16-byte aligned");
  const b2::CommView v = b2::make_view(comm);
  // Decode-sized calls (a rank owns at most kMaxCtas rows): one CTA per owned row, one
  // 8-element vector per thread (dim / 8 threads), at least 64 CTAs for the copy-out.
  // Prefill-sized calls: CTAs of dim / 32 threads (four vectors per thread, so a row's 8
  // sources x 4 loads are in flight per thread), as many as can be resident at once, each
  // looping over its share of the owned rows; rows then proceed in parallel instead of
  // one per CTA of a 128-CTA grid.  Every CTA of the grid must be resident together: part
  // C waits for rows that other ranks' CTAs reduce, so a CTA that never got an SM could
  // stall every rank until the timeout.
  int grid, threads;
  bool multi;
  if (R <= b2::kMaxCtas) {
    grid = R < 64 ? 64 : R;
    threads = 64;
    while (threads < 512 && threads < dim / 8) threads *= 2;
    multi = false;
  } else {
    threads = 64;
    while (threads < 512 && threads * 32 < dim) threads *= 2;
    // resident CTAs per SM: the smaller of the two instantiations the grid may run
    int occ = 1 << 30;
    const void* fns[2] = {
        dtype == B2_BF16 ? (const void*)b2::allreduce_rmsnorm_sharded_kernel<__nv_bfloat16, true>
                         : (const void*)b2::allreduce_rmsnorm_sharded_kernel<float, true>,
        dtype == B2_BF16 ? (const void*)b2::allreduce_rmsnorm_sharded_kernel<__nv_bfloat16, false>
                         : (const void*)b2::allreduce_rmsnorm_sharded_kernel<float, false>};
    for (const void* fn : fns) {
      int o = 0;
      B2_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, fn, threads, 0));
      occ = o < occ ? o : occ;
    }
    const long resident = (long)(occ < 1 ? 1 : occ) * b2::sm_count();
    grid = (int)(R < resident ? R : resident);
    multi = R > grid;
  }
  if (dtype == B2_BF16)
    B2_TRY_CUDA(b2::launch_pdl(multi ? b2::allreduce_rmsnorm_sharded_kernel<__nv_bfloat16, true>
                                     : b2::allreduce_rmsnorm_sharded_kernel<__nv_bfloat16, false>,
                               dim3(grid), dim3(threads), 0, stream, v, rows, R, dim, h_slice, norm_w, eps,
                               (__nv_bfloat16*)y, timeout_ns, status));
  else
    B2_TRY_CUDA(b2::launch_pdl(multi ? b2::allreduce_rmsnorm_sharded_kernel<float, true>
                                     : b2::allreduce_rmsnorm_sharded_kernel<float, false>,
                               dim3(grid), dim3(threads), 0, stream, v, rows, R, dim, h_slice, norm_w, eps, (float*)y,
                               timeout_ns, status));
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

}  // extern "C"
