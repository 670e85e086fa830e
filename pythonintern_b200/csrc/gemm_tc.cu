// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA.
//
// y[m, n] = sum_k x[m, k] * w[n, k] for the column/row-parallel linears of the
// decoder layer (engine/tensor_parallel/layers.py:83, :152; attention.py:156-158,
// :232; mlp.py:80-85).  Decode makes M (tokens) small and N (features) large, so
// the kernel runs "swap-AB": the packed weight tile (128 feature rows) is the MMA's
// A operand and the token tile (BN = 16..256 rows) is its B operand, giving
// D[feature, token] = W . X^T in TMEM.  Per CTA:
//
//   warp 0 / lane 0 : TMA producer, STAGES-deep ring of {W 128x64, X BNx64} bf16
//                     tiles, 128-byte swizzle, no multicast
//   warp 1 / lane 0 : MMA issuer, tcgen05.mma.cta_group::1.kind::f16, M=128,
//                     N=BN, K=16 x4 per stage; tcgen05.commit frees each stage
//   all 4 warps      : epilogue, tcgen05.ld 32x32b rows -> registers -> global
//
// Split-K over CTAs spreads skinny decode GEMMs over all SMs: every split writes
// its float32 partial tile to the workspace, and the last split of a tile (atomic
// counter) sums them and runs the epilogue.  Epilogues: plain store (optional
// bias, bf16 or f32 output), grouped q|k|v segments, and SwiGLU, where each
// 128-row A tile is 64 gate rows + the 64 matching up rows and the epilogue
// writes silu(g) * u.  Every wait is bounded by %globaltimer; a timeout raises
// B2_DEV_PIPE_TIMEOUT, drains the copies in flight, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "gemm.cuh"

namespace b2 {
namespace tc {

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BK = 64;   // K elements per stage = one 128-byte swizzle atom
constexpr int kThreads = 128;
constexpr int kMaxSegs = 3;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s bound on any pipeline wait

struct Params {
  int M, nkb, kb_per_split, splits;
  int n_tiles, m_tiles, nseg;
  int seg_tile_start[kMaxSegs + 1];
  int seg_n[kMaxSegs];
  int seg_col[kMaxSegs];
  int epi;
  const float* bias;
  void* y;
  int64_t ldy;
  int y_dtype;
  float* ws;
  int* counters;
  int32_t* status;
};

// ------------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: true on completion, false after kWaitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t bound_ns = kWaitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0 && globaltimer_ns() - t0 > bound_ns) return false;
  }
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns; waits for the load before returning.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row core
// groups 1024 bytes apart (stride byte offset), sm_100 descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                   // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset
  d |= (uint64_t)1 << 46;                   // descriptor version
  d |= (uint64_t)2 << 61;                   // SWIZZLE_128B
  return d;
}
// Instruction descriptor, kind::f16: bf16 A and B, f32 accumulator, both K-major.
__host__ __device__ constexpr uint32_t instr_desc_bf16(int m, int n) {
  return (1u << 4)                        // D format: f32
         | (1u << 7)                      // A format: bf16
         | (1u << 10)                     // B format: bf16
         | ((uint32_t)(n >> 3) << 17)     // N / 8
         | ((uint32_t)(m >> 4) << 24);    // M / 16
}

template <int BN>
struct Cfg {
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024;
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW0,
                   const __grid_constant__ CUtensorMap tmW1, const __grid_constant__ CUtensorMap tmW2,
                   const Params p) {
  using C = Cfg<BN>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int s_last;

  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int tile = blockIdx.x, mt = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Constant indices only: a dynamically indexed parameter array would be copied
  // to local memory.
  int seg = 0;
  if (p.nseg > 1 && tile >= p.seg_tile_start[1]) seg = 1;
  if (p.nseg > 2 && tile >= p.seg_tile_start[2]) seg = 2;
  const int local_tile = tile - (seg == 0 ? p.seg_tile_start[0] : seg == 1 ? p.seg_tile_start[1] : p.seg_tile_start[2]);
  const int seg_n = seg == 0 ? p.seg_n[0] : seg == 1 ? p.seg_n[1] : p.seg_n[2];
  const int seg_col = seg == 0 ? p.seg_col[0] : seg == 1 ? p.seg_col[1] : p.seg_col[2];
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(p.nkb, kb0 + p.kb_per_split);
  const int nk = kb1 - kb0;
  const int m0 = mt * BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  int issued = 0;
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    for (int i = 0; i < nk; ++i) {
      const int st = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      if (!mbar_wait(&empty_bar[st], ph ^ 1u)) {
        raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
        break;
      }
      uint8_t* sa = smem + (size_t)st * C::STAGE_BYTES;
      uint8_t* sb = sa + C::A_BYTES;
      mbar_arrive_expect_tx(&full_bar[st], C::STAGE_BYTES);
      const int kx = (kb0 + i) * BK;
      if (p.epi == kEpiSwiglu) {
        tma_load_2d(sa, &tmW0, &full_bar[st], kx, local_tile * 64, pol_w);
        tma_load_2d(sa + C::A_BYTES / 2, &tmW1, &full_bar[st], kx, local_tile * 64, pol_w);
      } else if (seg == 0) {  // descriptors are addressed in param space, never copied
        tma_load_2d(sa, &tmW0, &full_bar[st], kx, local_tile * BM, pol_w);
      } else if (seg == 1) {
        tma_load_2d(sa, &tmW1, &full_bar[st], kx, local_tile * BM, pol_w);
      } else {
        tma_load_2d(sa, &tmW2, &full_bar[st], kx, local_tile * BM, pol_w);
      }
      tma_load_2d(sb, &tmX, &full_bar[st], kx, m0, pol_x);
      ++issued;
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = instr_desc_bf16(BM, BN);
    for (int i = 0; i < nk; ++i) {
      const int st = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      if (!mbar_wait(&full_bar[st], ph)) {
        raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
        break;
      }
      tc_fence_after();
      const uint32_t a_addr = smem_u32(smem + (size_t)st * C::STAGE_BYTES);
      const uint64_t adesc = smem_desc_sw128(a_addr);
      const uint64_t bdesc = smem_desc_sw128(a_addr + C::A_BYTES);
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk)  // +32 bytes along K per MMA = +2 in the address field
        umma_bf16(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
      umma_commit(&empty_bar[st]);
    }
    umma_commit(&done_bar);
  }
  __syncwarp();

  // ---------------- epilogue
  // Block-uniform verdict so that the epilogue's barriers are reached by all threads.
  const bool done = __syncthreads_and(mbar_wait(&done_bar, 0)) != 0;
  tc_fence_after();
  if (!done && threadIdx.x == 0) raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
  const int r = warp * 32 + lane;  // accumulator row = TMEM lane
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  const int M = p.M;

  if (done && p.splits == 1) {
    if (p.epi == kEpiStore) {
      const int n = local_tile * BM + r;
      const bool nok = n < seg_n;
      const int64_t col = (int64_t)seg_col + n;
      const float bv = (nok && p.bias) ? p.bias[col] : 0.f;
      for (int c0 = 0; c0 < BN && m0 + c0 < M; c0 += 16) {
        float v[16];
        tmem_ld16(trow + c0, v);
        if (nok) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c0 + j;
            if (m < M) st_dyn(p.y, p.y_dtype, (int64_t)m * p.ldy + col, v[j] + bv);
          }
        }
      }
    } else {
      // SwiGLU: TMEM lanes 0-63 hold gate rows, 64-127 the matching up rows.
      float* su = reinterpret_cast<float*>(smem);  // [BN][64], pipeline buffers are idle now
      if (warp >= 2) {
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(trow + c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) su[(c0 + j) * 64 + (r - 64)] = v[j];
        }
      }
      __syncthreads();
      if (warp < 2) {
        const int n = local_tile * 64 + r;
        const bool nok = n < p.seg_n[0];
        for (int c0 = 0; c0 < BN && m0 + c0 < M; c0 += 16) {
          float v[16];
          tmem_ld16(trow + c0, v);
          if (nok) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = m0 + c0 + j;
              if (m < M) st_dyn(p.y, p.y_dtype, (int64_t)m * p.ldy + n, silu_f32(v[j]) * su[(c0 + j) * 64 + r]);
            }
          }
        }
      }
    }
  } else if (done) {
    // Split-K: publish this split's float32 tile, the last split reduces.
    const int64_t tile_elems = (int64_t)BM * BN;
    const int64_t slot = (int64_t)tile * p.m_tiles + mt;
    float* mine = p.ws + ((int64_t)split * p.n_tiles * p.m_tiles + slot) * tile_elems;
    for (int c0 = 0; c0 < BN && m0 + c0 < M; c0 += 16) {
      float v[16];
      tmem_ld16(trow + c0, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) mine[(int64_t)(c0 + j) * BM + r] = v[j];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      int* ctr = p.counters + slot;
      const int prev = atomicAdd(ctr, 1);
      s_last = prev == p.splits - 1;
      if (s_last) *ctr = 0;
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      const int64_t split_stride = (int64_t)p.n_tiles * p.m_tiles * tile_elems;
      const float* base = p.ws + slot * tile_elems;
      const int ncols = min(BN, M - m0);
      const int nsplit = p.splits;
      if (p.epi == kEpiStore) {
        // Each warp reduces whole token columns (128 contiguous floats = 32 lanes x float4),
        // 4 columns per pass with every split's loads issued before any store.
        const int r4 = lane * 4;
        const int n0 = local_tile * BM + r4;
        float bv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) bv[e] = (p.bias && n0 + e < seg_n) ? p.bias[seg_col + n0 + e] : 0.f;
        for (int cb = warp * 4; cb < ncols; cb += 16) {
          float4 acc[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int sp = 0; sp < nsplit; ++sp) {
            const float* src = base + sp * split_stride + r4;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              if (cb + u < ncols) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(src + (int64_t)(cb + u) * BM));
                acc[u].x += v.x; acc[u].y += v.y; acc[u].z += v.z; acc[u].w += v.w;
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (cb + u >= ncols) continue;
            const int64_t rowoff = (int64_t)(m0 + cb + u) * p.ldy + seg_col;
            const float vals[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (n0 + e < seg_n) st_dyn(p.y, p.y_dtype, rowoff + n0 + e, vals[e] + bv[e]);
          }
        }
      } else {
        // SwiGLU: lanes 0-15 / 16-31 take two token columns; each lane holds 4 gate rows
        // (TMEM lanes 0-63 of the tile) and the matching 4 up rows (64-127).
        const int half = lane >> 4;
        const int r4 = (lane & 15) * 4;
        const int n0 = local_tile * 64 + r4;
        for (int cb = warp * 2 + half; cb < ncols; cb += 8) {
          float4 gs = make_float4(0.f, 0.f, 0.f, 0.f), us = gs;
          for (int sp = 0; sp < nsplit; ++sp) {
            const float* src = base + sp * split_stride + (int64_t)cb * BM + r4;
            const float4 gv = __ldcg(reinterpret_cast<const float4*>(src));
            const float4 uv = __ldcg(reinterpret_cast<const float4*>(src + 64));
            gs.x += gv.x; gs.y += gv.y; gs.z += gv.z; gs.w += gv.w;
            us.x += uv.x; us.y += uv.y; us.z += uv.z; us.w += uv.w;
          }
          const int64_t rowoff = (int64_t)(m0 + cb) * p.ldy;
          const float g4[4] = {gs.x, gs.y, gs.z, gs.w}, u4[4] = {us.x, us.y, us.z, us.w};
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (n0 + e < seg_n) st_dyn(p.y, p.y_dtype, rowoff + n0 + e, silu_f32(g4[e]) * u4[e]);
        }
      }
    }
  }

  // ---------------- teardown
  if (warp == 0 && lane == 0) {
    // Copies still in flight after an aborted pipeline land before the CTA exits.
    for (int st = 0; st < STAGES && st < issued; ++st) {
      const int last_i = st + ((issued - 1 - st) / STAGES) * STAGES;
      mbar_wait(&full_bar[st], (uint32_t)(last_i / STAGES) & 1u, 100000000ull);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2D bf16 tensor map: `rows` rows of `k` elements, `row_bytes` apart; box = 64 x box_rows.
static int make_map(CUtensorMap* m, const void* ptr, uint64_t k, uint64_t rows, uint64_t row_bytes,
                    uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(B2_ECUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {k, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B2_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return B2_OK;
}

struct Plan {
  int BN, m_tiles, n_tiles, nkb, splits, kbps;
};

static Plan make_plan(int M, int n_tiles, int K) {
  Plan pl{};
  pl.BN = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  pl.m_tiles = (M + pl.BN - 1) / pl.BN;
  pl.n_tiles = n_tiles;
  pl.nkb = (K + BK - 1) / BK;
  // Cost in bytes moved through one SM on the critical path: every wave streams
  // kbps stages; with split-K each CTA also writes a float32 partial tile and the
  // last CTA of a tile reads all of them back.
  const int sms = sm_count();
  const long units = (long)n_tiles * pl.m_tiles;
  const long stage = (long)(BM + pl.BN) * BK * 2;
  const long partial = (long)BM * pl.BN * 4;
  long best_cost = -1;
  for (int s = 1; s <= 16 && s <= pl.nkb; ++s) {
    const int kbps = (pl.nkb + s - 1) / s;
    const int s_eff = (pl.nkb + kbps - 1) / kbps;
    const long waves = (units * s_eff + sms - 1) / sms;
    const long cost = waves * (kbps * stage + (s_eff > 1 ? partial : 0)) + (s_eff > 1 ? s_eff * partial : 0);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      pl.splits = s_eff;
      pl.kbps = kbps;
    }
  }
  return pl;
}

// Workspace layout: a FIXED-size counter region (so that launches of different tile
// counts never see each other's partial tiles as counters), then the partial tiles.
constexpr size_t kCounterSlots = 65536;
constexpr size_t kCounterBytes = kCounterSlots * sizeof(int);

static size_t plan_ws_bytes(const Plan& pl) {
  if (pl.splits <= 1) return 0;
  const size_t units = (size_t)pl.n_tiles * pl.m_tiles;
  return kCounterBytes + (size_t)pl.splits * units * BM * pl.BN * sizeof(float);
}

template <int BN>
static int launch(const CUtensorMap& mx, const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& w2,
                  const Params& p, dim3 grid, cudaStream_t s) {
  using C = Cfg<BN>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    B2_TRY_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
    attr_set[dev] = true;
  }
  gemm_tc_kernel<BN><<<grid, kThreads, C::SMEM, s>>>(mx, w0, w1, w2, p);
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

}  // namespace tc

static int tc_tiles(const GemmSeg* segs, int nseg, int epi, int* starts) {
  int total = 0;
  for (int i = 0; i < nseg; ++i) {
    starts[i] = total;
    total += epi == kEpiSwiglu ? (segs[0].n + 63) / 64 : (segs[i].n + tc::BM - 1) / tc::BM;
    if (epi == kEpiSwiglu) break;
  }
  starts[epi == kEpiSwiglu ? 1 : nseg] = total;
  return total;
}

size_t gemm_tc_workspace_bytes(int M, int n_total, int K, int epi) {
  // Upper bound over segmentations of n_total into up to three parts.
  const int base = epi == kEpiSwiglu ? (n_total + 63) / 64 : (n_total + tc::BM - 1) / tc::BM;
  size_t best = 0;
  for (int extra = 0; extra <= (epi == kEpiSwiglu ? 0 : 2); ++extra) {
    const size_t b = tc::plan_ws_bytes(tc::make_plan(M, base + extra, K));
    if (b > best) best = b;
  }
  return best;
}

bool gemm_tc_supported(const void* x, int64_t ldx, int K, const GemmSeg* segs, int nseg) {
  if (K % 8 != 0 || (ldx % 8) != 0 || ((uintptr_t)x % 16) != 0) return false;
  for (int i = 0; i < nseg; ++i)
    if (((uintptr_t)segs[i].w % 16) != 0) return false;
  return true;
}

int gemm_tc(const void* x, int64_t ldx, int M, int K, const GemmSeg* segs, int nseg, int epi,
            const float* bias, void* y, int64_t ldy, int y_dtype, void* ws, size_t ws_bytes,
            int32_t* status, cudaStream_t s) {
  B2_CHECK_ARG(nseg >= 1 && nseg <= tc::kMaxSegs, "gemm_tc: bad segment count");
  B2_CHECK_ARG(gemm_tc_supported(x, ldx, K, segs, nseg),
               "gemm_tc: needs K %% 8 == 0, 16-byte aligned rows (K=%d ldx=%lld)", K, (long long)ldx);
  tc::Params p{};
  int starts[tc::kMaxSegs + 1] = {0, 0, 0, 0};
  const int n_tiles = tc_tiles(segs, nseg, epi, starts);
  const tc::Plan pl = tc::make_plan(M, n_tiles, K);
  B2_CHECK_ARG(pl.m_tiles <= 65535, "gemm_tc: M=%d too large", M);
  const size_t need = tc::plan_ws_bytes(pl);
  if (need > 0) {
    B2_CHECK_ARG(ws && ws_bytes >= need, "gemm_tc: workspace of %zu bytes needed, %zu given", need, ws_bytes);
  }
  p.M = M;
  p.nkb = pl.nkb;
  p.kb_per_split = pl.kbps;
  p.splits = pl.splits;
  p.n_tiles = n_tiles;
  p.m_tiles = pl.m_tiles;
  p.nseg = epi == kEpiSwiglu ? 1 : nseg;
  for (int i = 0; i <= tc::kMaxSegs; ++i) p.seg_tile_start[i] = starts[i];
  for (int i = 0; i < nseg; ++i) {
    p.seg_n[i] = segs[i].n;
    p.seg_col[i] = segs[i].col_off;
  }
  p.epi = epi;
  p.bias = bias;
  p.y = y;
  p.ldy = ldy;
  p.y_dtype = y_dtype;
  if (need > 0) {
    B2_CHECK_ARG((size_t)pl.n_tiles * pl.m_tiles <= tc::kCounterSlots, "gemm_tc: too many tiles for split-K");
    p.counters = reinterpret_cast<int*>(ws);
    p.ws = reinterpret_cast<float*>(static_cast<char*>(ws) + tc::kCounterBytes);
  }
  p.status = status;

  CUtensorMap mx, mw[3];
  const uint32_t wrows = epi == kEpiSwiglu ? 64 : tc::BM;
  int rc = tc::make_map(&mx, x, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, (uint32_t)pl.BN);
  if (rc) return rc;
  for (int i = 0; i < 3; ++i) {
    const GemmSeg& sg = segs[i < nseg ? i : 0];
    rc = tc::make_map(&mw[i], sg.w, (uint64_t)K, (uint64_t)sg.n, (uint64_t)K * 2, wrows);
    if (rc) return rc;
  }
  dim3 grid(n_tiles, pl.m_tiles, pl.splits);
  switch (pl.BN) {
    case 16: return tc::launch<16>(mx, mw[0], mw[1], mw[2], p, grid, s);
    case 32: return tc::launch<32>(mx, mw[0], mw[1], mw[2], p, grid, s);
    case 64: return tc::launch<64>(mx, mw[0], mw[1], mw[2], p, grid, s);
    case 128: return tc::launch<128>(mx, mw[0], mw[1], mw[2], p, grid, s);
    default: return tc::launch<256>(mx, mw[0], mw[1], mw[2], p, grid, s);
  }
}

}  // namespace b2
