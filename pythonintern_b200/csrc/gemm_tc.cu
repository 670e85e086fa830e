// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA.
//
// y[m, n] = sum_k x[m, k] * w[n, k] for the column/row-parallel linears of the
// decoder layer (engine/tensor_parallel/layers.py:83, :152; attention.py:156-158,
// :232; mlp.py:80-85).  Decode makes M (tokens) small and N (features) large, so
// the kernel runs "swap-AB": the packed weight tile (128 feature rows) is the MMA's
// A operand and the token tile (BN = 16..256 rows) is its B operand, giving
// D[feature, token] = W . X^T in TMEM.  Per CTA:
//
//   warp 0 / lane 0 : TMA producer, STAGES-deep ring of {W 128x64 (gate and up for
//                     SwiGLU), X BNx64} bf16 tiles, 128-byte swizzle, no multicast
//   warp 1 / lane 0 : MMA issuer, tcgen05.mma.cta_group::1.kind::f16, M=128,
//                     N=BN, K=16 x4 per stage; tcgen05.commit frees each stage
//   epilogue warps   : tcgen05.ld 32x32b rows -> registers -> global
//
// Two kernels.  gemm_tc_kernel is persistent (one CTA per SM walking the tiles, TMEM
// accumulators double-buffered so a tile's epilogue overlaps the next mainloop; a
// uniform split-K fallback whose last CTA per tile reduces).  gemm_tc_cluster_kernel
// splits K over a thread-block cluster of s CTAs per tile for the skinny decode GEMMs:
// partials go through an L2 workspace and one cluster barrier, each CTA reducing 1/s of
// the token columns.  Epilogues: plain store (optional bias, bf16 or f32 output, or the
// reduce-scatter push of the tensor-parallel row-parallel GEMM), grouped q|k|v segments
// (optionally with RoPE + the paged KV write), SwiGLU (gate and up accumulators in two
// TMEM column ranges, silu(g) * u), the deferred RMSNorm producer (residual add, h * w,
// tile sums of h^2) and consumer (row scale).  Every wait is bounded by %globaltimer; a
// timeout raises B2_DEV_PIPE_TIMEOUT, drains the copies in flight, frees TMEM and returns.
#include <cuda.h>
#include <map>
#include <mutex>
#include <tuple>
#include <cudaTypedefs.h>

#include "gemm.cuh"
#include "tc_ptx.cuh"

namespace b2 {
namespace tc {

constexpr int BM = 128;  // weight rows per tile (MMA M)
constexpr int BK = 64;   // K elements per stage = one 128-byte swizzle atom
constexpr int kThreads = 192;  // 6 warps: producer, MMA, 4 epilogue
// Cluster split-K kernel: producer, MMA, 8 warps that publish the partial tile (two per
// TMEM lane quarter) and 2 more; all 12 warps share the reduction, which is bound by
// the number of L2 loads in flight.
constexpr int kThreadsCl = 384;
constexpr int kMaxSegs = 3;

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
  const unsigned long long* sc_table;  // reduce-scatter destinations (sc_world > 0)
  const unsigned int* sc_epoch;
  int sc_R, sc_src, sc_world;
  int vec4;  // output columns in aligned groups of 4: store 4 elements per instruction
  // Deferred RMSNorm at world size 1 (see b2_linear_residual_norm).  Consumer (row_ss set):
  // output row m is scaled by rsqrt(sum_j row_ss[m * n_ss + j] * ss_scale + ss_eps) ahead of
  // the epilogue (both SwiGLU halves).  Producer (res_h set, split-K cluster path only):
  // h[m, n] += acc, z[m, n] = bf16(h * norm_w[n]), ss_out[m * ss_tiles + tile] = sum of h^2
  // over the tile's 128 columns; nothing else is stored.
  const float* row_ss;
  int n_ss;
  float ss_scale, ss_eps;
  float* res_h;
  int64_t ldh;
  const float* norm_w;
  __nv_bfloat16* z;
  int64_t ldz;
  float* ss_out;
  int ss_tiles;
  // Fused RoPE + paged KV write (q|k|v GEMM, head_dim 128): tile h < nq is q head h, then
  // the k heads, then the v heads; nothing else is stored.
  int rope;
  int nq, nkv;
  const int64_t* rope_pos;
  const int64_t* store_pos;
  const int32_t* table_index;
  const int32_t* tables;
  int table_stride, num_blocks, block_size, max_seq_len;
  const float* cos_t;
  const float* sin_t;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t layer_off;
};

// rsqrt(mean square + eps) of row m from its per-tile partial sums, summed in tile order
// (every caller computes the identical value); eight loads in flight per round.
__device__ __forceinline__ float row_inv(const Params& p, int64_t m) {
  const float* q = p.row_ss + m * p.n_ss;
  float s = 0.f;
  int j = 0;
  for (; j + 8 <= p.n_ss; j += 8) {
    float a[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) a[u] = q[j + u];
#pragma unroll
    for (int u = 0; u < 8; ++u) s += a[u];
  }
  for (; j < p.n_ss; ++j) s += q[j];
  return rsqrtf(s * p.ss_scale + p.ss_eps);
}

__device__ __forceinline__ void store_out(const Params& p, int64_t m, int64_t col, float v) {
  int64_t idx;
  void* base = out_base(p.y, p.y_dtype, p.ldy, p.sc_table, p.sc_epoch, p.sc_R, p.sc_src, p.sc_world, m, col, &idx);
  st_dyn(base, p.y_dtype, idx, v);
}
// Four consecutive output columns col..col+3 of row m (p.vec4: col % 4 == 0, aligned rows):
// one 8-byte (bf16) or 16-byte (float32) store, which keeps peer-memory writes whole.
__device__ __forceinline__ void store_out4(const Params& p, int64_t m, int64_t col, const float (&v)[4]) {
  int64_t idx;
  void* base = out_base(p.y, p.y_dtype, p.ldy, p.sc_table, p.sc_epoch, p.sc_R, p.sc_src, p.sc_world, m, col, &idx);
  if (p.y_dtype == B2_BF16) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&lo);
    o.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(base) + idx) = o;
  } else {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + idx) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// Named barrier over the four epilogue warps only (the producer and MMA warps keep running).
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// AND of `pred` over the four epilogue warps (a barrier among them, like epilogue_sync).
__device__ __forceinline__ bool epilogue_all(bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)pred)
      : "memory");
  return out != 0;
}


template <int BN, bool SWIGLU>
struct Cfg {
  static constexpr uint32_t A_BYTES = (SWIGLU ? 2 : 1) * BM * BK * 2;  // gate (+ up) weight tiles
  static constexpr uint32_t B_BYTES = BN * BK * 2;                      // activation tile
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES;
  static constexpr uint32_t ACC_COLS = (SWIGLU ? 2 : 1) * BN;           // TMEM columns per accumulator
  static constexpr int NBUF = 2 * ACC_COLS <= 512 ? 2 : 1;              // double-buffered accumulators
  static constexpr uint32_t TMEM_COLS = NBUF * ACC_COLS < 32 ? 32 : NBUF * ACC_COLS;
  static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024;
  static_assert(STAGES >= 2, "pipeline too shallow");
  static_assert((TMEM_COLS & (TMEM_COLS - 1)) == 0 && TMEM_COLS <= 512, "TMEM allocation must be a power of 2");
};

// Unit u -> (split, tile, m tile); the splits of one tile are consecutive units, so
// persistent CTAs working side by side finish a tile's splits at about the same time.
struct Unit {
  int split, tile, mt;
};
__device__ __forceinline__ Unit decode_unit(const Params& p, int u) {
  Unit w;
  w.split = u % p.splits;
  const int rest = u / p.splits;
  w.tile = rest % p.n_tiles;
  w.mt = rest / p.n_tiles;
  return w;
}

// Persistent warp-specialised kernel: warp 0 = TMA producer, warp 1 = MMA issuer and
// TMEM owner, warps 2-5 = epilogue (TMEM lane quarter = warp % 4).
template <int BN, bool SWIGLU>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW0,
                   const __grid_constant__ CUtensorMap tmW1, const __grid_constant__ CUtensorMap tmW2,
                   const Params p) {
  using C = Cfg<BN, SWIGLU>;
  constexpr int STAGES = C::STAGES;
  constexpr int NBUF = C::NBUF;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full[NBUF];
  __shared__ __align__(8) uint64_t acc_empty[NBUF];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int s_last;
  __shared__ float s_inv[BN];  // deferred RMSNorm: per-token scale of the current unit
  __shared__ void* s_row[BN];  // per token of the current unit: its output row (after the scatter)

  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = p.n_tiles * p.m_tiles * p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  pdl_wait();  // barrier set-up and TMEM allocation overlap the previous kernel's tail
  pdl_trigger();

  if (warp == 0) {
    // ---------------- TMA producer (one lane)
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const Unit w = decode_unit(p, u);
        int seg = 0;
        if (p.nseg > 1 && w.tile >= p.seg_tile_start[1]) seg = 1;
        if (p.nseg > 2 && w.tile >= p.seg_tile_start[2]) seg = 2;
        const int local_tile = w.tile - (seg == 0 ? p.seg_tile_start[0] : seg == 1 ? p.seg_tile_start[1]
                                                                                    : p.seg_tile_start[2]);
        const int kb0 = w.split * p.kb_per_split;
        const int kb1 = min(p.nkb, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int st = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!mbar_wait(&empty_bar[st], ph ^ 1u)) {
            raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
            ok = false;
            break;
          }
          uint8_t* sa = smem + (size_t)st * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          mbar_arrive_expect_tx(&full_bar[st], C::STAGE_BYTES);
          const int kx = kb * BK;
          if (SWIGLU) {
            tma_load_2d(sa, &tmW0, &full_bar[st], kx, local_tile * BM, pol_w);
            tma_load_2d(sa + BM * BK * 2, &tmW1, &full_bar[st], kx, local_tile * BM, pol_w);
          } else if (seg == 0) {  // descriptors are addressed in param space, never copied
            tma_load_2d(sa, &tmW0, &full_bar[st], kx, local_tile * BM, pol_w);
          } else if (seg == 1) {
            tma_load_2d(sa, &tmW1, &full_bar[st], kx, local_tile * BM, pol_w);
          } else {
            tma_load_2d(sa, &tmW2, &full_bar[st], kx, local_tile * BM, pol_w);
          }
          tma_load_2d(sb, &tmX, &full_bar[st], kx, w.mt * BN, pol_x);
        }
      }
      // Copies still in flight (only after an aborted pipeline) land before the CTA exits.
      for (int st = 0; st < STAGES && st < it; ++st) {
        const int last_i = st + ((it - 1 - st) / STAGES) * STAGES;
        mbar_wait(&full_bar[st], (uint32_t)(last_i / STAGES) & 1u, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer: the whole warp runs the control code (the descriptors stay
    // in uniform registers), one elected lane issues.  The tensor cores queue only about one
    // MMA ahead, so the next stage's barrier is tested while this stage's MMAs go out
    // (peek), and its wait costs nothing when the copy has already landed.
    constexpr uint32_t idesc = instr_desc_bf16(BM, BN);
    int it = 0, j = 0;
    bool ok = true;
    Peek pk{0u, 0u, false};
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++j) {
      const Unit w = decode_unit(p, u);
      const int buf = j % NBUF;
      const uint32_t acc = tmem + (uint32_t)(buf * C::ACC_COLS);
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_empty[buf], ((uint32_t)(j / NBUF) & 1u) ^ 1u))) {
        if (lane == 0) raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
        break;
      }
      tc_fence_after();
      const int kb0 = w.split * p.kb_per_split;
      const int kb1 = min(p.nkb, kb0 + p.kb_per_split);
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int st = it % STAGES;
        const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
        if (!__all_sync(0xffffffffu, wait_peeked(pk, &full_bar[st], ph))) {
          if (lane == 0) raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + (size_t)st * C::STAGE_BYTES);
        const uint64_t adesc = smem_desc_sw128(a_addr);
        const uint64_t bdesc = smem_desc_sw128(a_addr + C::A_BYTES);
        const uint32_t first = kb == kb0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {  // +32 bytes along K per MMA = +2 in the address field
          if (elect_one()) umma_bf16(acc, adesc + 2 * kk, bdesc + 2 * kk, idesc, (first && kk == 0) ? 0u : 1u);
          if (kk == 0)  // the next stage (of this unit or the next), while this one's MMAs run
            peek(pk, &full_bar[(it + 1) % STAGES], (uint32_t)((it + 1) / STAGES) & 1u);
        }
        if (SWIGLU) {
          const uint64_t udesc = smem_desc_sw128(a_addr + BM * BK * 2);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            if (elect_one()) umma_bf16(acc + BN, udesc + 2 * kk, bdesc + 2 * kk, idesc, (first && kk == 0) ? 0u : 1u);
        }
        if (elect_one()) umma_commit(&empty_bar[st]);
      }
      if (elect_one()) umma_commit(&acc_full[buf]);
    }
    // Every MMA issued by the elected lane has completed once drain_bar fires.
    if (elect_one()) umma_commit(&drain_bar);
    mbar_wait(&drain_bar, 0, 100000000ull);
    __syncwarp();
  } else {
    // ---------------- epilogue warps 2-5
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // accumulator row = TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const int M = p.M;
    int j = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++j) {
      const Unit w = decode_unit(p, u);
      int seg = 0;
      if (p.nseg > 1 && w.tile >= p.seg_tile_start[1]) seg = 1;
      if (p.nseg > 2 && w.tile >= p.seg_tile_start[2]) seg = 2;
      const int local_tile = w.tile - (seg == 0 ? p.seg_tile_start[0] : seg == 1 ? p.seg_tile_start[1]
                                                                                  : p.seg_tile_start[2]);
      const int seg_n = seg == 0 ? p.seg_n[0] : seg == 1 ? p.seg_n[1] : p.seg_n[2];
      const int seg_col = seg == 0 ? p.seg_col[0] : seg == 1 ? p.seg_col[1] : p.seg_col[2];
      const int buf = j % NBUF;
      const uint32_t acc = tmem + lane_base + (uint32_t)(buf * C::ACC_COLS);
      const int m0 = w.mt * BN;
      const int ncols = min(BN, M - m0);
      const int n = local_tile * BM + r;
      const bool nok = n < seg_n;
      // Uniform verdict: the split-K path below meets at named barriers.
      const bool done = epilogue_all(mbar_wait(&acc_full[buf], (uint32_t)(j / NBUF) & 1u));
      if (!done) {
        if (lane == 0) raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
        break;
      }
      tc_fence_after();
      if (p.splits == 1) {
        const int64_t col = (int64_t)seg_col + n;
        const float bv = (nok && p.bias) ? p.bias[col] : 0.f;
        // Row addresses once per unit: the tensor-parallel scatter's owner rank and slot
        // (a division and two loads) would otherwise be recomputed for every element.
        for (int c = threadIdx.x - 64; c < ncols; c += 128) {
          int64_t idx;
          void* base = out_base(p.y, p.y_dtype, p.ldy, p.sc_table, p.sc_epoch, p.sc_R, p.sc_src, p.sc_world,
                                m0 + c, 0, &idx);
          s_row[c] = static_cast<char*>(base) + idx * (p.y_dtype == B2_BF16 ? 2 : 4);
          if (p.row_ss) s_inv[c] = row_inv(p, m0 + c);
        }
        epilogue_sync();
        for (int c0 = 0; c0 < ncols; c0 += 16) {
          float v[16];
          tmem_ld16(acc + c0, v);
          if (p.row_ss) {
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] *= s_inv[min(c0 + e, ncols - 1)];
          }
          if (SWIGLU) {
            float uv[16];
            tmem_ld16(acc + BN + c0, uv);
            if (p.row_ss) {
#pragma unroll
              for (int e = 0; e < 16; ++e) uv[e] *= s_inv[min(c0 + e, ncols - 1)];
            }
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = silu_f32(v[e]) * uv[e];
          }
          if (nok) {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c0 + e < ncols) st_dyn(s_row[c0 + e], p.y_dtype, (size_t)col, v[e] + bv);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        epilogue_sync();  // s_row / s_inv are rewritten by the next unit
      } else {
        // Split-K: publish this split's float32 tile ([column][128 rows], gate then up for
        // SwiGLU), release TMEM, and let the last split of the tile reduce.
        constexpr int PARTS = SWIGLU ? 2 : 1;
        const int64_t tile_elems = (int64_t)PARTS * BM * BN;
        const int64_t slot = (int64_t)w.tile * p.m_tiles + w.mt;
        float* mine = p.ws + ((int64_t)w.split * p.n_tiles * p.m_tiles + slot) * tile_elems;
        for (int c0 = 0; c0 < ncols; c0 += 16) {
#pragma unroll
          for (int part = 0; part < PARTS; ++part) {
            float v[16];
            tmem_ld16(acc + part * BN + c0, v);
#pragma unroll
            for (int e = 0; e < 16; ++e) mine[((int64_t)part * BN + c0 + e) * BM + r] = v[e];
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        __threadfence();
        epilogue_sync();
        if (threadIdx.x == 64) {
          int* ctr = p.counters + slot;
          const int prev = atomicAdd(ctr, 1);
          s_last = prev == p.splits - 1;
          if (s_last) *ctr = 0;
        }
        epilogue_sync();
        if (s_last) {
          __threadfence();
          if (p.row_ss) {
            for (int c = threadIdx.x - 64; c < ncols; c += 128) s_inv[c] = row_inv(p, m0 + c);
            epilogue_sync();
          }
          const int64_t split_stride = (int64_t)p.n_tiles * p.m_tiles * tile_elems;
          const float* base = p.ws + slot * tile_elems;
          // Each epilogue warp reduces whole token columns: 32 lanes x float4 = 128 rows.
          const int r4 = lane * 4;
          const int nb = local_tile * BM + r4;
          float bv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) bv[e] = (!SWIGLU && p.bias && nb + e < seg_n) ? p.bias[seg_col + nb + e] : 0.f;
          for (int c = quarter; c < ncols; c += 4) {
            float4 g4 = make_float4(0.f, 0.f, 0.f, 0.f), u4 = g4;
            for (int sp = 0; sp < p.splits; ++sp) {
              const float* src = base + sp * split_stride + (int64_t)c * BM + r4;
              const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
              g4.x += a.x; g4.y += a.y; g4.z += a.z; g4.w += a.w;
              if (SWIGLU) {
                const float4 b = __ldcg(reinterpret_cast<const float4*>(src + (int64_t)BN * BM));
                u4.x += b.x; u4.y += b.y; u4.z += b.z; u4.w += b.w;
              }
            }
            const float inv = p.row_ss ? s_inv[c] : 1.f;
            const float gv[4] = {g4.x * inv, g4.y * inv, g4.z * inv, g4.w * inv};
            const float uv[4] = {u4.x * inv, u4.y * inv, u4.z * inv, u4.w * inv};
            float val[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) val[e] = SWIGLU ? silu_f32(gv[e]) * uv[e] : gv[e] + bv[e];
            if (p.vec4 && nb + 3 < seg_n) {
              store_out4(p, m0 + c, seg_col + nb, val);
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                if (nb + e < seg_n) store_out(p, m0 + c, seg_col + nb + e, val[e]);
            }
          }
        }
        epilogue_sync();  // s_last is rewritten by the next unit
      }
    }
  }

  // ---------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------
// Split-K over a thread-block cluster.  One cluster per output tile, one CTA per K split
// (cluster rank = split).  After its mainloop each CTA writes its float32 partial tile
// from TMEM to its own workspace region; after one cluster barrier (release / acquire at
// cluster scope), CTA k sums column slice k of every CTA's partial, read from L2 in split
// order, and stores that slice.  The cluster only guarantees that the CTAs of a tile are
// resident together, so the barrier cannot wait on a CTA that was never scheduled.
constexpr int kMaxClusterSplits = 8;  // portable cluster size: split-K of at most 8
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
template <int BN, bool SWIGLU>
__global__ void __launch_bounds__(kThreadsCl, 1)
    gemm_tc_cluster_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW0,
                           const __grid_constant__ CUtensorMap tmW1, const __grid_constant__ CUtensorMap tmW2,
                           const Params p) {
  using C = Cfg<BN, SWIGLU>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full;
  __shared__ uint32_t tmem_slot;

  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = (int)cluster_rank();
  const int tile = blockIdx.x / p.splits;
  const int mt = blockIdx.y;
  int seg = 0;
  if (p.nseg > 1 && tile >= p.seg_tile_start[1]) seg = 1;
  if (p.nseg > 2 && tile >= p.seg_tile_start[2]) seg = 2;
  const int local_tile = tile - (seg == 0 ? p.seg_tile_start[0] : seg == 1 ? p.seg_tile_start[1] : p.seg_tile_start[2]);
  const int seg_n = seg == 0 ? p.seg_n[0] : seg == 1 ? p.seg_n[1] : p.seg_n[2];
  const int seg_col = seg == 0 ? p.seg_col[0] : seg == 1 ? p.seg_col[1] : p.seg_col[2];
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(p.nkb, kb0 + p.kb_per_split);
  const int m0 = mt * BN;
  const int ncols = min(BN, p.M - m0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  pdl_wait();  // barrier set-up and TMEM allocation overlap the previous kernel's tail
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int it = 0;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int st = it % STAGES;
        const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
        if (!mbar_wait(&empty_bar[st], ph ^ 1u)) {
          raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
          break;
        }
        uint8_t* sa = smem + (size_t)st * C::STAGE_BYTES;
        mbar_arrive_expect_tx(&full_bar[st], C::STAGE_BYTES);
        const int kx = kb * BK;
        if (SWIGLU) {
          tma_load_2d(sa, &tmW0, &full_bar[st], kx, local_tile * BM, pol_w);
          tma_load_2d(sa + BM * BK * 2, &tmW1, &full_bar[st], kx, local_tile * BM, pol_w);
        } else if (seg == 0) {
          tma_load_2d(sa, &tmW0, &full_bar[st], kx, local_tile * BM, pol_w);
        } else if (seg == 1) {
          tma_load_2d(sa, &tmW1, &full_bar[st], kx, local_tile * BM, pol_w);
        } else {
          tma_load_2d(sa, &tmW2, &full_bar[st], kx, local_tile * BM, pol_w);
        }
        tma_load_2d(sa + C::A_BYTES, &tmX, &full_bar[st], kx, m0, pol_x);
      }
      for (int st = 0; st < STAGES && st < it; ++st) {
        const int last_i = st + ((it - 1 - st) / STAGES) * STAGES;
        mbar_wait(&full_bar[st], (uint32_t)(last_i / STAGES) & 1u, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // MMA issuer: warp-uniform control code, one elected lane issues, the next stage's
    // barrier tested while this stage's MMAs go out (as in gemm_tc_kernel).
    constexpr uint32_t idesc = instr_desc_bf16(BM, BN);
    int it = 0;
    Peek pk{0u, 0u, false};
    for (int kb = kb0; kb < kb1; ++kb, ++it) {
      const int st = it % STAGES;
      const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
      if (!__all_sync(0xffffffffu, wait_peeked(pk, &full_bar[st], ph))) {
        if (lane == 0) raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
        break;
      }
      tc_fence_after();
      const uint32_t a_addr = smem_u32(smem + (size_t)st * C::STAGE_BYTES);
      const uint64_t adesc = smem_desc_sw128(a_addr);
      const uint64_t bdesc = smem_desc_sw128(a_addr + C::A_BYTES);
      const uint32_t first = kb == kb0 ? 1u : 0u;
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        if (elect_one()) umma_bf16(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (first && kk == 0) ? 0u : 1u);
        if (kk == 0 && kb + 1 < kb1) peek(pk, &full_bar[(it + 1) % STAGES], (uint32_t)((it + 1) / STAGES) & 1u);
      }
      if (SWIGLU) {
        const uint64_t udesc = smem_desc_sw128(a_addr + BM * BK * 2);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          if (elect_one()) umma_bf16(tmem + BN, udesc + 2 * kk, bdesc + 2 * kk, idesc, (first && kk == 0) ? 0u : 1u);
      }
      if (elect_one()) umma_commit(&empty_bar[st]);
    }
    if (elect_one()) umma_commit(&acc_full);
    __syncwarp();
  }

  // Publish this CTA's float32 partial tile ([part][column][128 rows]) to its workspace
  // region straight from TMEM; after the cluster barrier every CTA reduces its slice of
  // token columns over the partials of all the cluster's CTAs, in split order, from L2.
  constexpr int PARTS = SWIGLU ? 2 : 1;
  constexpr int64_t PART_ELEMS = (int64_t)PARTS * BN * BM;
  const int64_t cta_lin = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
  if (warp >= 2 && warp < 10) {
    const int quarter = warp & 3;          // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;      // alternate 16-column chunks between two warps
    const int r = quarter * 32 + lane;
    const uint32_t acc = tmem + ((uint32_t)(quarter * 32) << 16);
    float* mine = p.ws + cta_lin * PART_ELEMS;
    const bool done = mbar_wait(&acc_full, 0);
    if (!done && lane == 0) raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
    tc_fence_after();
#pragma unroll
    for (int part = 0; part < PARTS; ++part) {
      for (int c0 = 16 * half; c0 < ncols; c0 += 32) {
        float v[16];
        tmem_ld16(acc + part * BN + c0, v);
#pragma unroll
        for (int e = 0; e < 16; ++e) mine[(part * BN + c0 + e) * BM + r] = done ? v[e] : 0.f;
      }
    }
  }
  cluster_sync_all();  // release / acquire at cluster scope: every partial of the cluster is visible

  const float* part0 = p.ws + (cta_lin - split) * PART_ELEMS;  // split 0 of this tile
  const int per = (ncols + p.splits - 1) / p.splits;
  const int c_lo = split * per, c_hi = min(ncols, c_lo + per);
  __shared__ float s_inv[BN];  // deferred RMSNorm consumer: scale of each token of this slice
  __shared__ int s_pos[BN];    // fused RoPE: position of each token (-1: out of range)
  __shared__ int64_t s_slot[BN];  // fused RoPE: element offset of its KV slot (-1: out of range)
  if (p.row_ss || p.rope) {
    for (int t = threadIdx.x; t < c_hi - c_lo; t += kThreadsCl) {
      const int tok = m0 + c_lo + t;
      if (p.row_ss) s_inv[t] = row_inv(p, tok);
      if (p.rope) {
        const int64_t pos = p.rope_pos[tok];
        const int64_t ps = p.store_pos ? p.store_pos[tok] : pos;
        const int row = p.table_index ? p.table_index[tok] : tok;
        const bool pos_ok = pos >= 0 && pos < p.max_seq_len;
        int64_t blk = -1;
        if (ps >= 0 && (ps / p.block_size) < p.table_stride)
          blk = p.tables[(int64_t)row * p.table_stride + ps / p.block_size];
        const bool slot_ok = blk >= 0 && blk < p.num_blocks;
        if (tile == 0 && !(pos_ok && slot_ok)) raise_status(p.status, B2_DEV_RANGE);
        s_pos[t] = pos_ok ? (int)pos : -1;
        s_slot[t] = slot_ok ? p.layer_off + ((blk * p.block_size + ps % p.block_size) * p.nkv) * (int64_t)BM : -1;
      }
    }
    __syncthreads();
  }
  constexpr int VPC = BM / 4;  // float4 vectors per token column
  constexpr int U = SWIGLU ? 1 : 2;  // vectors per thread whose loads are all issued first
  const int nvec = (c_hi > c_lo ? c_hi - c_lo : 0) * VPC;
  for (int i0 = threadIdx.x; i0 < nvec; i0 += U * kThreadsCl) {
    float4 ga[U][kMaxClusterSplits], ua[U][SWIGLU ? kMaxClusterSplits : 1];
    float4 hres[U], wres[U];  // deferred RMSNorm producer: residual and norm weight, loaded up front
    float4 crope[U], srope[U];  // fused RoPE: cos / sin of the token's position, loaded up front
#pragma unroll
    for (int h = 0; h < U; ++h) {
      const int i = i0 + h * kThreadsCl;
      if (i >= nvec) continue;
      const float* src = part0 + (int64_t)(c_lo + i / VPC) * BM + (i % VPC) * 4;
      if (!SWIGLU && p.rope && tile < p.nq + p.nkv) {
        const int pos = s_pos[i / VPC];
        if (pos >= 0) {
          crope[h] = *reinterpret_cast<const float4*>(p.cos_t + (int64_t)pos * BM + (i % VPC) * 4);
          srope[h] = *reinterpret_cast<const float4*>(p.sin_t + (int64_t)pos * BM + (i % VPC) * 4);
        }
      }
      if (!SWIGLU && p.res_h) {
        const int64_t ncol = (int64_t)seg_col + local_tile * BM + (i % VPC) * 4;
        hres[h] = *reinterpret_cast<const float4*>(p.res_h + (int64_t)(m0 + c_lo + i / VPC) * p.ldh + ncol);
        wres[h] = *reinterpret_cast<const float4*>(p.norm_w + ncol);
      }
#pragma unroll
      for (int q = 0; q < kMaxClusterSplits; ++q) {
        if (q < p.splits) {
          ga[h][q] = __ldcg(reinterpret_cast<const float4*>(src + q * PART_ELEMS));
          if (SWIGLU) ua[h][q] = __ldcg(reinterpret_cast<const float4*>(src + q * PART_ELEMS + (int64_t)BN * BM));
        }
      }
    }
#pragma unroll
    for (int h = 0; h < U; ++h) {
      const int i = i0 + h * kThreadsCl;
      if (i >= nvec) continue;
      const int c = c_lo + i / VPC;
      const int r4 = (i % VPC) * 4;
      float4 g4 = make_float4(0.f, 0.f, 0.f, 0.f), u4 = g4;
#pragma unroll
      for (int q = 0; q < kMaxClusterSplits; ++q) {
        if (q < p.splits) {
          g4.x += ga[h][q].x; g4.y += ga[h][q].y; g4.z += ga[h][q].z; g4.w += ga[h][q].w;
          if (SWIGLU) {
            u4.x += ua[h][q].x; u4.y += ua[h][q].y; u4.z += ua[h][q].z; u4.w += ua[h][q].w;
          }
        }
      }
      const int nb = local_tile * BM + r4;
      const float inv = p.row_ss ? s_inv[c - c_lo] : 1.f;
      const float gv[4] = {g4.x * inv, g4.y * inv, g4.z * inv, g4.w * inv};
      const float uv[4] = {u4.x * inv, u4.y * inv, u4.z * inv, u4.w * inv};
      float val[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float bv = (!SWIGLU && p.bias && nb + e < seg_n) ? p.bias[seg_col + nb + e] : 0.f;
        val[e] = SWIGLU ? silu_f32(gv[e]) * uv[e] : gv[e] + bv;
      }
      if (!SWIGLU && p.rope) {
        // Fused RoPE + paged KV write: the GEMM output rounded to bf16 (as the q|k|v buffer
        // would hold it) is rotated with the same two-rounding formula as rope_kv_write_kernel;
        // the rotate-half partner of columns d..d+3 sits in lane ^ 16 of this warp.
        const int head = tile;
        const int tok = m0 + c;
        float x[4], xp[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = __bfloat162float(__float2bfloat16_rn(val[e]));
#pragma unroll
        for (int e = 0; e < 4; ++e) xp[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
        if (s_pos[c - c_lo] < 0) continue;
        const int64_t slot_off = s_slot[c - c_lo];
        const bool slot_ok = slot_off >= 0;
        float o[4];
        if (head < p.nq + p.nkv) {
          const bool lower = r4 < BM / 2;
          const float ct[4] = {crope[h].x, crope[h].y, crope[h].z, crope[h].w};
          const float st[4] = {srope[h].x, srope[h].y, srope[h].z, srope[h].w};
#pragma unroll
          for (int e = 0; e < 4; ++e)  // lower: x1*cos - x2*sin;  upper: x2*cos + x1*sin
            o[e] = __fadd_rn(__fmul_rn(x[e], ct[e]), __fmul_rn(lower ? -xp[e] : xp[e], st[e]));
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) o[e] = x[e];
        }
        __nv_bfloat16* dst;
        if (head < p.nq) {
          dst = p.q_out + ((int64_t)tok * p.nq + head) * BM + r4;
        } else {
          if (!slot_ok) continue;
          dst = head < p.nq + p.nkv ? p.k_cache + slot_off + (int64_t)(head - p.nq) * BM + r4
                                    : p.v_cache + slot_off + (int64_t)(head - p.nq - p.nkv) * BM + r4;
        }
        __nv_bfloat162 lo = __floats2bfloat162_rn(o[0], o[1]), hi = __floats2bfloat162_rn(o[2], o[3]);
        uint2 ov;
        ov.x = *reinterpret_cast<uint32_t*>(&lo);
        ov.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(dst) = ov;
        continue;
      }
      if (!SWIGLU && p.res_h) {
        // Deferred RMSNorm producer: residual add, h * w in bf16, and the tile's sum of h^2
        // for this token (the warp's 32 lanes hold the tile's 128 columns).
        const int64_t ncol = (int64_t)seg_col + nb;
        float4 hv = hres[h];
        hv.x += val[0]; hv.y += val[1]; hv.z += val[2]; hv.w += val[3];
        *reinterpret_cast<float4*>(p.res_h + (int64_t)(m0 + c) * p.ldh + ncol) = hv;
        const float4 wv = wres[h];
        __nv_bfloat162 lo = __floats2bfloat162_rn(hv.x * wv.x, hv.y * wv.y);
        __nv_bfloat162 hi = __floats2bfloat162_rn(hv.z * wv.z, hv.w * wv.w);
        uint2 zo;
        zo.x = *reinterpret_cast<uint32_t*>(&lo);
        zo.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(p.z + (int64_t)(m0 + c) * p.ldz + ncol) = zo;
        const float sq = warp_sum(hv.x * hv.x + hv.y * hv.y + hv.z * hv.z + hv.w * hv.w);
        if (lane == 0) p.ss_out[(int64_t)(m0 + c) * p.ss_tiles + (seg_col + local_tile * BM) / BM] = sq;
        continue;
      }
      if (p.vec4 && nb + 3 < seg_n) {
        store_out4(p, m0 + c, seg_col + nb, val);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (nb + e < seg_n) store_out(p, m0 + c, seg_col + nb + e, val[e]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
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

// The cluster split-K path serves token tiles of up to 128 columns.
#define BN_FITS_CLUSTER(bn, swiglu) ((bn) <= 128)

struct Plan {
  int BN, m_tiles, n_tiles, nkb, splits, kbps, ctas;
  bool cluster;  // split-K over one thread-block cluster per tile (else the persistent kernel)
};

// Clusters of s CTAs of the split-K kernel that can be resident at once on this device
// (the GPCs' SM counts decide how clusters of 3, 5, 6 or 7 pack); cached per device.
template <int BN, bool SWIGLU>
static int max_active_clusters_t(int s) {
  using C = Cfg<BN, SWIGLU>;
  if (cudaFuncSetAttribute(gemm_tc_cluster_kernel<BN, SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)C::SMEM) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)s, 1, 1);
  cfg.blockDim = dim3(kThreadsCl, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)s;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_cluster_kernel<BN, SWIGLU>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

static int max_active_clusters(int BN, bool swiglu, int s) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const auto key = std::make_tuple(dev, BN, swiglu ? 1 : 0, s);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  switch (BN) {
    case 16: n = swiglu ? max_active_clusters_t<16, true>(s) : max_active_clusters_t<16, false>(s); break;
    case 32: n = swiglu ? max_active_clusters_t<32, true>(s) : max_active_clusters_t<32, false>(s); break;
    case 64: n = swiglu ? max_active_clusters_t<64, true>(s) : max_active_clusters_t<64, false>(s); break;
    default: n = swiglu ? max_active_clusters_t<128, true>(s) : max_active_clusters_t<128, false>(s); break;
  }
  cache[key] = n;
  return n;
}

// Launch plan.  When the output has at least half as many 128-row tiles as there are
// SMs, the persistent kernel without split-K streams best (measured on B200 over the
// decode shapes: M = 1..128 tokens; q|k|v, o_proj, gate|up, down of the 8B shape).
// Otherwise K is split over a thread-block cluster of s CTAs per tile, with the largest
// s <= 8 (the portable cluster size) for which every tile's cluster is resident at once
// (one wave, asked of the occupancy calculator).  The cluster's CTAs exchange float32
// partials through an L2 workspace and one cluster barrier, each reducing 1/s of the
// token columns; an exchange through distributed shared memory, or a barrier built from
// L2 atomics instead of the cluster barrier, measured about twice as slow.  The
// persistent split-K path (last CTA of a tile reduces) remains for token tiles wider
// than 128 (BN = 256).
static Plan make_plan(int M, int n_tiles, int K, bool swiglu) {
  Plan pl{};
  // 129-512 tokens: 256-wide token tiles when they alone give the persistent kernel at
  // least half a wave (no split-K); otherwise 128-wide tiles, which keep the split-K
  // cluster path and the fused epilogues instead of the 256-wide tile's single-CTA
  // split-K reduction (measured on B200 at 240 decode rows, 8B shape: q|k|v 58 -> 32 us,
  // o_proj 52 -> 17 us at TP=1; gate|up, 112 weight tiles, stays at 256: 76 vs 85 us).
  const int sms = sm_count();
  if (M <= 128) {
    pl.BN = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  } else if (M <= 512) {
    const long t256 = (long)n_tiles * ((M + 255) / 256);
    pl.BN = 2 * t256 >= sms ? 256 : 128;
  } else {
    pl.BN = 256;
  }
  pl.m_tiles = (M + pl.BN - 1) / pl.BN;
  pl.n_tiles = n_tiles;
  pl.nkb = (K + BK - 1) / BK;
  const long tiles = (long)n_tiles * pl.m_tiles;
  pl.splits = 1;
  pl.kbps = pl.nkb;
  pl.cluster = false;
  if (2 * tiles < sms && BN_FITS_CLUSTER(pl.BN, swiglu)) {
    const int s_max = (int)std::min<long>(std::min<long>(kMaxClusterSplits, pl.nkb), sms / tiles);
    for (int s = s_max; s >= 2; --s) {
      const int kbps = (pl.nkb + s - 1) / s;
      const int s_eff = (pl.nkb + kbps - 1) / kbps;
      if (s_eff != s) continue;
      if (max_active_clusters(pl.BN, swiglu, s) < tiles) continue;
      pl.splits = s;
      pl.kbps = kbps;
      pl.cluster = true;
      break;
    }
  }
  if (!pl.cluster && 2 * tiles < sms) {
    for (int s : {8, 4, 2}) {
      if (tiles * s > sms || s > pl.nkb) continue;
      const int kbps = (pl.nkb + s - 1) / s;
      const int s_eff = (pl.nkb + kbps - 1) / kbps;
      if (s_eff < 2) continue;
      pl.splits = s_eff;
      pl.kbps = kbps;
      break;
    }
  }
  const long units = tiles * pl.splits;
  pl.ctas = pl.cluster ? (int)units : (int)(units < sms ? units : sms);
  return pl;
}

// Workspace layout: a FIXED-size counter region (so that launches of different tile
// counts never see each other's partial tiles as counters), then the partial tiles.
constexpr size_t kCounterSlots = 65536;
constexpr size_t kCounterBytes = kCounterSlots * sizeof(int);

static size_t plan_ws_bytes(const Plan& pl, bool swiglu) {
  if (pl.splits <= 1) return 0;
  const size_t tiles = (size_t)pl.n_tiles * pl.m_tiles;
  return kCounterBytes + (size_t)pl.splits * tiles * (swiglu ? 2 : 1) * BM * pl.BN * sizeof(float);
}

template <int BN, bool SWIGLU>
static int launch(const CUtensorMap& mx, const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& w2,
                  const Params& p, int ctas, cudaStream_t s) {
  using C = Cfg<BN, SWIGLU>;
  static bool attr_set[64] = {false};
  int dev = 0;
  B2_TRY_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    B2_TRY_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)C::SMEM));
    attr_set[dev] = true;
  }
  B2_TRY_CUDA(launch_pdl((gemm_tc_kernel<BN, SWIGLU>), dim3(ctas), dim3(kThreads), C::SMEM, s, mx, w0, w1, w2, p));
  return B2_OK;
}

template <int BN, bool SWIGLU>
static int launch_cluster(const CUtensorMap& mx, const CUtensorMap& w0, const CUtensorMap& w1,
                          const CUtensorMap& w2, const Params& p, cudaStream_t s) {
  using C = Cfg<BN, SWIGLU>;
  static bool attr_set[64] = {false};
  int dev = 0;
  B2_TRY_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    B2_TRY_CUDA(cudaFuncSetAttribute(gemm_tc_cluster_kernel<BN, SWIGLU>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.n_tiles * p.splits), (unsigned)p.m_tiles, 1);
  cfg.blockDim = dim3(kThreadsCl, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)p.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see pdl_wait()
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  B2_TRY_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc_cluster_kernel<BN, SWIGLU>, mx, w0, w1, w2, p));
  return B2_OK;
}

template <bool SWIGLU>
static int launch_cluster_bn(int BN, const CUtensorMap& mx, const CUtensorMap* mw, const Params& p,
                             cudaStream_t s) {
  switch (BN) {
    case 16: return launch_cluster<16, SWIGLU>(mx, mw[0], mw[1], mw[2], p, s);
    case 32: return launch_cluster<32, SWIGLU>(mx, mw[0], mw[1], mw[2], p, s);
    case 64: return launch_cluster<64, SWIGLU>(mx, mw[0], mw[1], mw[2], p, s);
    default: return launch_cluster<128, SWIGLU>(mx, mw[0], mw[1], mw[2], p, s);
  }
}

template <bool SWIGLU>
static int launch_bn(int BN, const CUtensorMap& mx, const CUtensorMap* mw, const Params& p, int ctas,
                     cudaStream_t s) {
  switch (BN) {
    case 16: return launch<16, SWIGLU>(mx, mw[0], mw[1], mw[2], p, ctas, s);
    case 32: return launch<32, SWIGLU>(mx, mw[0], mw[1], mw[2], p, ctas, s);
    case 64: return launch<64, SWIGLU>(mx, mw[0], mw[1], mw[2], p, ctas, s);
    case 128: return launch<128, SWIGLU>(mx, mw[0], mw[1], mw[2], p, ctas, s);
    default: return launch<256, SWIGLU>(mx, mw[0], mw[1], mw[2], p, ctas, s);
  }
}

}  // namespace tc

static int tc_tiles(const GemmSeg* segs, int nseg, int epi, int* starts) {
  int total = 0;
  const int n_used = epi == kEpiSwiglu ? 1 : nseg;
  for (int i = 0; i < n_used; ++i) {
    starts[i] = total;
    total += (segs[i].n + tc::BM - 1) / tc::BM;
  }
  for (int i = n_used; i <= tc::kMaxSegs; ++i) starts[i] = total;
  return total;
}

size_t gemm_tc_workspace_bytes(int M, int n_total, int K, int epi) {
  // Upper bound over segmentations of n_total into up to three parts.
  const bool sw = epi == kEpiSwiglu;
  const int base = (n_total + tc::BM - 1) / tc::BM;
  size_t best = 0;
  for (int extra = 0; extra <= (sw ? 0 : 2); ++extra) {
    const size_t b = tc::plan_ws_bytes(tc::make_plan(M, base + extra, K, sw), sw);
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
            int32_t* status, cudaStream_t s, const Scatter* sc, const RowNorm* rn, const RopeKV* rk) {
  B2_CHECK_ARG(nseg >= 1 && nseg <= tc::kMaxSegs, "gemm_tc: bad segment count");
  B2_CHECK_ARG(gemm_tc_supported(x, ldx, K, segs, nseg),
               "gemm_tc: needs K %% 8 == 0, 16-byte aligned rows (K=%d ldx=%lld)", K, (long long)ldx);
  const bool sw = epi == kEpiSwiglu;
  tc::Params p{};
  int starts[tc::kMaxSegs + 1] = {0, 0, 0, 0};
  const int n_tiles = tc_tiles(segs, nseg, epi, starts);
  const tc::Plan pl = tc::make_plan(M, n_tiles, K, sw);
  const size_t need = tc::plan_ws_bytes(pl, sw);
  // the cluster kernel always exchanges partials through the workspace
  B2_CHECK_ARG(!pl.cluster || (pl.splits >= 2 && need > 0), "gemm_tc: split-K cluster plan without a workspace");
  if (need > 0) {
    B2_CHECK_ARG(ws && ws_bytes >= need, "gemm_tc: workspace of %zu bytes needed, %zu given", need, ws_bytes);
    B2_CHECK_ARG((size_t)pl.n_tiles * pl.m_tiles <= tc::kCounterSlots, "gemm_tc: too many tiles for split-K");
  }
  p.M = M;
  p.nkb = pl.nkb;
  p.kb_per_split = pl.kbps;
  p.splits = pl.splits;
  p.n_tiles = n_tiles;
  p.m_tiles = pl.m_tiles;
  p.nseg = sw ? 1 : nseg;
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
    p.counters = reinterpret_cast<int*>(ws);
    p.ws = reinterpret_cast<float*>(static_cast<char*>(ws) + tc::kCounterBytes);
  }
  p.status = status;
  {
    const size_t esz = y_dtype == B2_BF16 ? 2 : 4;
    bool v4 = ldy % 4 == 0 && (sc && sc->world > 0 ? true : ((uintptr_t)y % (4 * esz)) == 0);
    for (int i = 0; i < nseg; ++i) v4 = v4 && segs[i].col_off % 4 == 0 && segs[i].n % 4 == 0;
    p.vec4 = v4 ? 1 : 0;
  }
  if (rn && rn->row_ss) {
    B2_CHECK_ARG(rn->n_ss > 0, "gemm_tc: row norm needs n_ss > 0");
    p.row_ss = rn->row_ss;
    p.n_ss = rn->n_ss;
    p.ss_scale = rn->ss_scale;
    p.ss_eps = rn->ss_eps;
  }
  if (rn && rn->res_h) {
    if (!pl.cluster || sw || nseg != 1 || segs[0].n % tc::BM != 0 || !p.vec4 || y_dtype != B2_BF16)
      return fail(B2_ENOTSUP, "gemm_tc: residual-norm epilogue needs the split-K cluster plan");
    B2_CHECK_ARG(rn->norm_w && rn->z && rn->ss_out && rn->ldh % 4 == 0 && rn->ldz % 4 == 0 &&
                     ((uintptr_t)rn->res_h % 16) == 0 && ((uintptr_t)rn->norm_w % 16) == 0 &&
                     ((uintptr_t)rn->z % 8) == 0,
                 "gemm_tc: residual-norm buffers must be aligned (h, norm_w 16 B; z 8 B; strides % 4)");
    p.res_h = rn->res_h;
    p.ldh = rn->ldh;
    p.norm_w = rn->norm_w;
    p.z = static_cast<__nv_bfloat16*>(rn->z);
    p.ldz = rn->ldz;
    p.ss_out = rn->ss_out;
    p.ss_tiles = segs[0].n / tc::BM;
  }
  if (rk) {
    if (!pl.cluster || sw || nseg != 3 || y_dtype != B2_BF16)
      return fail(B2_ENOTSUP, "gemm_tc: fused RoPE epilogue needs the split-K cluster plan");
    B2_CHECK_ARG(segs[0].n == rk->nq * tc::BM && segs[1].n == rk->nkv * tc::BM && segs[2].n == rk->nkv * tc::BM,
                 "gemm_tc: fused RoPE needs head_dim 128 (one weight tile per head)");
    B2_CHECK_ARG(((uintptr_t)rk->q_out % 8) == 0 && ((uintptr_t)rk->k_cache % 8) == 0 &&
                     ((uintptr_t)rk->v_cache % 8) == 0 && ((uintptr_t)rk->cos_t % 16) == 0 &&
                     ((uintptr_t)rk->sin_t % 16) == 0,
                 "gemm_tc: fused RoPE buffers must be aligned (outputs 8 B, tables 16 B)");
    p.rope = 1;
    p.nq = rk->nq;
    p.nkv = rk->nkv;
    p.rope_pos = rk->rope_pos;
    p.store_pos = rk->store_pos;
    p.table_index = rk->table_index;
    p.tables = rk->tables;
    p.table_stride = rk->table_stride;
    p.num_blocks = rk->num_blocks;
    p.block_size = rk->block_size;
    p.max_seq_len = rk->max_seq_len;
    p.cos_t = rk->cos_t;
    p.sin_t = rk->sin_t;
    p.q_out = static_cast<__nv_bfloat16*>(rk->q_out);
    p.k_cache = static_cast<__nv_bfloat16*>(rk->k_cache);
    p.v_cache = static_cast<__nv_bfloat16*>(rk->v_cache);
    p.layer_off = rk->layer_off;
  }
  if (sc && sc->world > 0) {
    p.sc_table = sc->table;
    p.sc_epoch = sc->epoch;
    p.sc_R = sc->rows_per_rank;
    p.sc_src = sc->src;
    p.sc_world = sc->world;
  }

  CUtensorMap mx, mw[3];
  int rc = tc::make_map(&mx, x, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, (uint32_t)pl.BN);
  if (rc) return rc;
  for (int i = 0; i < 3; ++i) {
    const GemmSeg& sg = segs[i < nseg ? i : 0];
    rc = tc::make_map(&mw[i], sg.w, (uint64_t)K, (uint64_t)sg.n, (uint64_t)K * 2, tc::BM);
    if (rc) return rc;
  }
  if (pl.cluster)
    return sw ? tc::launch_cluster_bn<true>(pl.BN, mx, mw, p, s) : tc::launch_cluster_bn<false>(pl.BN, mx, mw, p, s);
  return sw ? tc::launch_bn<true>(pl.BN, mx, mw, p, pl.ctas, s) : tc::launch_bn<false>(pl.BN, mx, mw, p, pl.ctas, s);
}

}  // namespace b2
