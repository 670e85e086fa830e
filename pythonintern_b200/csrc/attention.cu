// Paged GQA attention for one query token per row over the block-table KV pool.
//
// Restates engine/model/attention.py:175-228 with engine/model/kv_cache.py:121-147:
// the reference gathers every sequence's K/V blocks into a dense zero-padded
// tensor, repeats the KV heads and runs softmax(q k^T / sqrt(d)) v.  Here the
// gather, GQA head sharing and the softmax are fused into one pass that reads
// each K/V row of the pool exactly once:
//
//  * grid = (splits, kv heads, rows); a CTA owns one (row, kv head) and a run of
//    KV blocks; its 4 warps interleave over the tokens of that run.
//  * Each lane group of HD/VEC lanes holds one token row as 16-byte vectors; the
//    REP = nq/nkv query heads that share the kv head are all scored against it,
//    so K and V are read once per kv head instead of once per q head.
//  * Online softmax in the log2 domain; partial states are merged across lane
//    groups (shuffles), warps (shared memory) and splits (workspace, merged by the
//    last CTA of the row to finish, found with an atomic counter).
//  * compat_pad reproduces the reference's unmasked zero padding
//    (attention.py:190-203): (max_ctx - ctx) extra keys with score 0 and value 0.
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"

namespace b2 {
int prefill_attention_tc(const void* q, int64_t ld_q, int n_rows, int nq, int nkv, const void* k_cache,
                         const void* v_cache, int64_t layer_off, int num_blocks, const int32_t* tables,
                         int table_stride, const int32_t* seq_start, const int32_t* seq_ctx0, int n_seqs,
                         float scale, void* out, int64_t ld_out, int32_t* status, cudaStream_t stream);

struct AttnParams {
  const void* q;
  int64_t ld_q;
  int n_rows, nq, nkv;
  const void* k_cache;
  const void* v_cache;
  int64_t layer_off;  // elements
  int block_size, num_blocks;
  const int32_t* tables;
  int table_stride;
  const int32_t* table_index;
  const int32_t* ctx_lens;
  int compat_pad;
  float scale_log2;  // softmax scale * log2(e)
  void* out;
  int64_t ld_out;
  float* ws_o;      // [rows, nq, splits, HD]
  float* ws_ml;     // [rows, nq, splits, 2]
  int* counters;    // [rows, nkv]
  int splits;
  int32_t* status;
};

constexpr int kAttnWarps = 4;

__device__ __forceinline__ float safe_exp2_diff(float a, float m) {
  return a == -INFINITY ? 0.f : exp2f(a - m);
}

// Merges the per-warp softmax states (sm_m/sm_l [nw][REP], sm_acc [nw][REP][HD]) of one
// (row, kv head, split), then either stores the output (one split) or publishes the
// split's state and lets the last split of (row, kv head) merge all of them.  Compat
// padding adds (max_ctx - ctx) keys of score 0 and value 0 to the final denominator.
template <typename T, int HD, int REP>
__device__ void attn_finalize(const AttnParams& p, const float* sm_m, const float* sm_l, const float* sm_acc,
                              int nw, int row, int g, int split, int ctx) {
  __shared__ float red[32];
  __shared__ int sm_flag;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps_block = blockDim.x >> 5;
  // Compat padding needs the longest context of the call.
  int max_ctx = ctx;
  if (p.compat_pad) {
    float mx = 0.f;
    for (int i = threadIdx.x; i < p.n_rows; i += blockDim.x) mx = fmaxf(mx, (float)p.ctx_lens[i]);
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    float all = red[0];
#pragma unroll
    for (int w = 1; w < nwarps_block; ++w) all = fmaxf(all, red[w]);
    max_ctx = (int)all;
  }
  const int npad = p.compat_pad ? max(0, max_ctx - ctx) : 0;

  T* outp = reinterpret_cast<T*>(p.out) + (int64_t)row * p.ld_out + (int64_t)g * REP * HD;
  const int64_t head0 = (int64_t)row * p.nq + g * REP;

  if (p.splits == 1) {
    for (int i = threadIdx.x; i < REP * HD; i += blockDim.x) {
      const int r = i / HD, d = i % HD;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < nw; ++w) M = fmaxf(M, sm_m[w * REP + r]);
      float L = 0.f, A = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < nw; ++w) {
          const float f = safe_exp2_diff(sm_m[w * REP + r], M);
          L += sm_l[w * REP + r] * f;
          A += sm_acc[(w * REP + r) * HD + d] * f;
        }
      }
      if (npad > 0) {
        const float Mp = fmaxf(M, 0.f);
        const float f = M == -INFINITY ? 0.f : exp2f(M - Mp);
        L = L * f + (float)npad * exp2f(-Mp);
        A = A * f;
      }
      outp[i] = from_f32<T>(L > 0.f ? A / L : 0.f);
    }
    return;
  }

  // Write this split's partial state, then let the last split of (row, g) merge.
  for (int i = threadIdx.x; i < REP * HD; i += blockDim.x) {
    const int r = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < nw; ++w) M = fmaxf(M, sm_m[w * REP + r]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < nw; ++w) {
        const float f = safe_exp2_diff(sm_m[w * REP + r], M);
        L += sm_l[w * REP + r] * f;
        A += sm_acc[(w * REP + r) * HD + d] * f;
      }
    }
    const int64_t h = head0 + r;
    p.ws_o[(h * p.splits + split) * HD + d] = A;
    if (d == 0) {
      p.ws_ml[(h * p.splits + split) * 2 + 0] = M;
      p.ws_ml[(h * p.splits + split) * 2 + 1] = L;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* ctr = p.counters + (int64_t)row * p.nkv + g;
    const int prev = atomicAdd(ctr, 1);
    const int last = prev == p.splits - 1;
    if (last) *ctr = 0;  // ready for the next launch
    sm_flag = last;
  }
  __syncthreads();
  if (!sm_flag) return;
  __threadfence();
  for (int i = threadIdx.x; i < REP * HD; i += blockDim.x) {
    const int r = i / HD, d = i % HD;
    const int64_t h = head0 + r;
    float M = -INFINITY;
    for (int s2 = 0; s2 < p.splits; ++s2) M = fmaxf(M, __ldcg(&p.ws_ml[(h * p.splits + s2) * 2]));
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
      for (int s2 = 0; s2 < p.splits; ++s2) {
        const float f = safe_exp2_diff(__ldcg(&p.ws_ml[(h * p.splits + s2) * 2]), M);
        L += __ldcg(&p.ws_ml[(h * p.splits + s2) * 2 + 1]) * f;
        A += __ldcg(&p.ws_o[(h * p.splits + s2) * HD + d]) * f;
      }
    }
    if (npad > 0) {
      const float Mp = fmaxf(M, 0.f);
      const float f = M == -INFINITY ? 0.f : exp2f(M - Mp);
      L = L * f + (float)npad * exp2f(-Mp);
      A = A * f;
    }
    outp[i] = from_f32<T>(L > 0.f ? A / L : 0.f);
  }
}

template <typename T, int HD, int REP>
__global__ void __launch_bounds__(kAttnWarps * 32) paged_attn_simt_kernel(AttnParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int VEC = 16 / sizeof(T);
  constexpr int LPT = HD / VEC;  // lanes per token row
  constexpr int G = 32 / LPT;    // token rows per warp step
  constexpr int CH = 4;          // tokens per lane group per chunk
  static_assert(LPT >= 1 && LPT <= 32 && (32 % LPT) == 0, "head_dim/vector mismatch");

  __shared__ float sm_m[kAttnWarps][REP], sm_l[kAttnWarps][REP];
  __shared__ float sm_acc[kAttnWarps][REP][HD];

  const int split = blockIdx.x, g = blockIdx.y, row = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / LPT, li = lane % LPT;
  const int ctx = max(0, p.ctx_lens[row]);
  const int bs = p.block_size;
  const int nblk = (ctx + bs - 1) / bs;
  const int bps = (nblk + p.splits - 1) / p.splits;
  const int t0 = min(ctx, split * bps * bs);
  const int t1 = min(ctx, (split + 1) * bps * bs);
  const int trow = p.table_index ? p.table_index[row] : row;
  const int32_t* table = p.tables + (int64_t)trow * p.table_stride;

  float q[REP][VEC];
#pragma unroll
  for (int r = 0; r < REP; ++r)
    load16_f32<T>(reinterpret_cast<const T*>(p.q) + (int64_t)row * p.ld_q + (int64_t)(g * REP + r) * HD + li * VEC, q[r]);

  float m[REP], l[REP], acc[REP][VEC];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[r][e] = 0.f;
  }

  const int64_t tok_stride = (int64_t)p.nkv * HD;
  const T* kbase = reinterpret_cast<const T*>(p.k_cache) + p.layer_off + (int64_t)g * HD + li * VEC;
  const T* vbase = reinterpret_cast<const T*>(p.v_cache) + p.layer_off + (int64_t)g * HD + li * VEC;

  for (int tb = t0 + warp * G; tb < t1; tb += kAttnWarps * G * CH) {
    float s[CH][REP];
    int64_t off[CH];
    bool ok[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int t = tb + c * kAttnWarps * G + sub;
      ok[c] = t < t1;
      off[c] = 0;
      if (ok[c]) {
        const int blk = table[t / bs];
        if (blk < 0 || blk >= p.num_blocks) {
          ok[c] = false;
          if (li == 0) raise_status(p.status, B2_DEV_RANGE);
        } else {
          off[c] = ((int64_t)blk * bs + (t % bs)) * tok_stride;
        }
      }
      float kv[VEC];
      if (ok[c]) {
        load16_f32<T>(kbase + off[c], kv);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) kv[e] = 0.f;
      }
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < VEC; ++e) d = fmaf(q[r][e], kv[e], d);
#pragma unroll
        for (int o = LPT / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        s[c][r] = ok[c] ? d * p.scale_log2 : -INFINITY;
      }
    }
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      float cm = s[0][r];
#pragma unroll
      for (int c = 1; c < CH; ++c) cm = fmaxf(cm, s[c][r]);
      const float mn = fmaxf(m[r], cm);
      if (mn == -INFINITY) {
#pragma unroll
        for (int c = 0; c < CH; ++c) s[c][r] = 0.f;
        continue;
      }
      const float corr = safe_exp2_diff(m[r], mn);
      l[r] *= corr;
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[r][e] *= corr;
      m[r] = mn;
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const float pr = safe_exp2_diff(s[c][r], mn);
        l[r] += pr;
        s[c][r] = pr;
      }
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      if (!ok[c]) continue;
      float vv[VEC];
      load16_f32<T>(vbase + off[c], vv);
#pragma unroll
      for (int r = 0; r < REP; ++r)
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[r][e] = fmaf(s[c][r], vv[e], acc[r][e]);
    }
  }

  // Merge lane groups of the warp (they hold disjoint tokens).
#pragma unroll
  for (int o = LPT; o < 32; o <<= 1) {
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[r], o);
      const float lo = __shfl_xor_sync(0xffffffffu, l[r], o);
      const float mn = fmaxf(m[r], mo);
      const float a = mn == -INFINITY ? 0.f : safe_exp2_diff(m[r], mn);
      const float b = mn == -INFINITY ? 0.f : safe_exp2_diff(mo, mn);
      l[r] = l[r] * a + lo * b;
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float ao = __shfl_xor_sync(0xffffffffu, acc[r][e], o);
        acc[r][e] = acc[r][e] * a + ao * b;
      }
      m[r] = mn;
    }
  }
  if (sub == 0) {
#pragma unroll
    for (int r = 0; r < REP; ++r) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) sm_acc[warp][r][li * VEC + e] = acc[r][e];
      if (li == 0) {
        sm_m[warp][r] = m[r];
        sm_l[warp][r] = l[r];
      }
    }
  }
  __syncthreads();

  attn_finalize<T, HD, REP>(p, &sm_m[0][0], &sm_l[0][0], &sm_acc[0][0][0], kAttnWarps, row, g, split, ctx);
}

// ---------------------------------------------------------------------------------------
// bf16 path: tensor-core (mma.sync m16n8k16) decode attention with cp.async pipelines.
//
// A CTA owns one (row, kv head, split); each of its 4 warps walks every 4th KV block
// of the CTA's run with its own STAGES-deep cp.async ring of whole blocks (16 token
// rows of K and of V for this kv head), so 12 blocks per CTA are in flight.  Rows are
// stored in shared memory with their 16-byte chunks XOR-swizzled by (row & 7), which
// keeps the ldmatrix reads below free of bank conflicts.  Per block a warp computes
//   S[16 x 16]  = Q[16 x HD] . K^T   (the REP <= 8 query heads of the group are rows
//                                     0..REP-1 of the 16-row MMA tile, 8 k-steps)
//   O[16 x HD] += P[16 x 16] . V      (P reused from the S accumulator registers)
// with an online softmax in the log2 domain.  The float32 softmax statistics, the
// per-warp merge and the split merge are shared with the SIMT kernel.
constexpr int kMmaWarps = 4;
constexpr int kMmaStages = 3;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}
// D = A . B + D, m16n8k16, bf16 inputs, f32 accumulators.
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int HD>
struct MmaCfg {
  static constexpr int ROWB = HD * 2;         // bytes of one token row of one kv head
  static constexpr int CHUNKS = ROWB / 16;    // 16-byte chunks per row
  static constexpr int SWZ = CHUNKS < 8 ? CHUNKS - 1 : 7;
  static constexpr int BLKB = 16 * ROWB;      // one K (or V) block
  static constexpr int STAGEB = 2 * BLKB;     // K + V
  static constexpr size_t SMEM = (size_t)kMmaWarps * kMmaStages * STAGEB;
};

template <int HD>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * MmaCfg<HD>::ROWB + ((chunk ^ (row & MmaCfg<HD>::SWZ)) << 4));
}

template <int HD, int REP, int W, int STAGES>
__global__ void __launch_bounds__(W * 32, W <= 4 ? 2 : 1) paged_attn_mma_kernel(AttnParams p) {
  pdl_wait();
  pdl_trigger();
  using C = MmaCfg<HD>;
  static_assert(REP <= 8, "the MMA tile holds up to 8 query heads per kv head");
  extern __shared__ __align__(128) uint8_t smem[];
  const int split = blockIdx.x, g = blockIdx.y, row = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int qr = lane >> 2, qt = lane & 3;  // MMA fragment row / column-pair of this lane
  const int ctx = max(0, p.ctx_lens[row]);
  const int bs = 16;
  const int nblk = (ctx + bs - 1) / bs;
  const int bps = (nblk + p.splits - 1) / p.splits;
  const int blk0 = min(nblk, split * bps);
  const int blk1 = min(nblk, blk0 + bps);
  const int trow = p.table_index ? p.table_index[row] : row;
  const int32_t* table = p.tables + (int64_t)trow * p.table_stride;
  const int n_w = blk1 - blk0 > warp ? (blk1 - blk0 - warp + W - 1) / W : 0;

  // Q fragments (A operand rows 0..7 = the REP heads, rows 8..15 = zero padding).
  uint32_t qa[HD / 16][2];
  {
    const __nv_bfloat16* qrow_ptr =
        reinterpret_cast<const __nv_bfloat16*>(p.q) + (int64_t)row * p.ld_q + (int64_t)(g * REP + qr) * HD;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      if (qr < REP) {
        qa[kk][0] = *reinterpret_cast<const uint32_t*>(qrow_ptr + kk * 16 + 2 * qt);
        qa[kk][1] = *reinterpret_cast<const uint32_t*>(qrow_ptr + kk * 16 + 8 + 2 * qt);
      } else {
        qa[kk][0] = qa[kk][1] = 0u;
      }
    }
  }

  const int64_t tok_stride_b = (int64_t)p.nkv * HD * 2;  // bytes between token rows of the pool
  const char* kbase = reinterpret_cast<const char*>(p.k_cache) + (p.layer_off + (int64_t)g * HD) * 2;
  const char* vbase = reinterpret_cast<const char*>(p.v_cache) + (p.layer_off + (int64_t)g * HD) * 2;
  const uint32_t wsm = smem_addr(smem) + (uint32_t)(warp * STAGES * C::STAGEB);

  // Issue the copies of this warp's i-th block into ring slot (i % STAGES); a block id
  // outside the pool is not copied, and the main loop skips that block.
  auto issue = [&](int i) {
    const int blk = table[blk0 + warp + i * W];
    if (blk < 0 || blk >= p.num_blocks) return;
    const uint32_t st = wsm + (uint32_t)((i % STAGES) * C::STAGEB);
    const int64_t blk_off = (int64_t)blk * bs * tok_stride_b;
#pragma unroll
    for (int q = lane; q < 16 * C::CHUNKS; q += 32) {
      const int r = q / C::CHUNKS, c = q % C::CHUNKS;
      const int64_t src = blk_off + r * tok_stride_b + c * 16;
      cp_async16(st + swz<HD>(r, c), kbase + src);
      cp_async16(st + C::BLKB + swz<HD>(r, c), vbase + src);
    }
  };

  float o[HD / 8][4];
#pragma unroll
  for (int d = 0; d < HD / 8; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // row qr statistics (per-lane partial l)

#pragma unroll
  for (int i = 0; i < STAGES - 1; ++i) {
    if (i < n_w) issue(i);
    cp_async_commit();
  }
  for (int i = 0; i < n_w; ++i) {
    if (i + STAGES - 1 < n_w) issue(i + STAGES - 1);
    cp_async_commit();
    cp_async_wait<STAGES - 1>();
    __syncwarp();
    const int bidx = blk0 + warp + i * W;
    const int blk = table[bidx];
    const bool blk_ok = blk >= 0 && blk < p.num_blocks;
    if (!blk_ok) {
      // Nothing was copied into this ring slot: skip the block entirely (scores AND the PV
      // product), so stale shared memory never reaches the output.
      if (lane == 0) raise_status(p.status, B2_DEV_RANGE);
      __syncwarp();
      continue;
    }
    const uint32_t ks = wsm + (uint32_t)((i % STAGES) * C::STAGEB);
    const uint32_t vs = ks + C::BLKB;

    // S = Q K^T over 16 tokens: two 8-token n-tiles.
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      // matrices: (tokens 0-7, dims lo), (tokens 0-7, dims hi), (tokens 8-15, lo), (tokens 8-15, hi)
      const int mrow = (lane & 7) + ((lane >> 4) << 3);
      const int mchunk = kk * 2 + ((lane >> 3) & 1);
      uint32_t b[4];
      ldsm_x4(ks + swz<HD>(mrow, mchunk), b);
      mma_bf16(s[0], qa[kk][0], 0u, qa[kk][1], 0u, b[0], b[1]);
      mma_bf16(s[1], qa[kk][0], 0u, qa[kk][1], 0u, b[2], b[3]);
    }
    // scale, mask, online softmax on row qr (accumulator elements 0, 1 of each n-tile)
    const int tbase = bidx * bs;
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = tbase + j * 8 + 2 * qt + e;
        const float v = (blk_ok && t < ctx) ? s[j][e] * p.scale_log2 : -INFINITY;
        s[j][e] = v;
        mx = fmaxf(mx, v);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float corr = safe_exp2_diff(m_run, m_new);
    float pv[2][2];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) pv[j][e] = m_new == -INFINITY ? 0.f : safe_exp2_diff(s[j][e], m_new);
    l_run = l_run * corr + (pv[0][0] + pv[0][1] + pv[1][0] + pv[1][1]);
    m_run = m_new;
#pragma unroll
    for (int d = 0; d < HD / 8; ++d) {
      o[d][0] *= corr;
      o[d][1] *= corr;
    }
    // P as the A operand (rows 8..15 zero), O += P V
    const uint32_t pa0 = pack_bf16(pv[0][0], pv[0][1]);
    const uint32_t pa2 = pack_bf16(pv[1][0], pv[1][1]);
#pragma unroll
    for (int d = 0; d < HD / 8; d += 2) {
      // matrices: (tokens 0-7, dims 8d), (tokens 8-15, dims 8d), (tokens 0-7, 8d+8), (tokens 8-15, 8d+8)
      const int mrow = (lane & 7) + (((lane >> 3) & 1) << 3);
      const int mchunk = d + (lane >> 4);
      uint32_t b[4];
      ldsm_x4_trans(vs + swz<HD>(mrow, mchunk), b);
      mma_bf16(o[d], pa0, 0u, pa2, 0u, b[0], b[1]);
      mma_bf16(o[d + 1], pa0, 0u, pa2, 0u, b[2], b[3]);
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  __syncthreads();  // the rings are idle; reuse them for the merge arrays

  float* sm_m = reinterpret_cast<float*>(smem);
  float* sm_l = sm_m + W * REP;
  float* sm_acc = sm_l + W * REP;
  if (qr < REP) {
    if (qt == 0) {
      sm_m[warp * REP + qr] = m_run;
      sm_l[warp * REP + qr] = l_run;
    }
#pragma unroll
    for (int d = 0; d < HD / 8; ++d) {
      sm_acc[(warp * REP + qr) * HD + d * 8 + 2 * qt] = o[d][0];
      sm_acc[(warp * REP + qr) * HD + d * 8 + 2 * qt + 1] = o[d][1];
    }
  }
  __syncthreads();
  attn_finalize<__nv_bfloat16, HD, REP>(p, sm_m, sm_l, sm_acc, W, row, g, split, ctx);
}

// ---------------------------------------------------------------------------------------
// Causal varlen prefill attention (bf16, mma.sync m16n8k16 over the paged pool).
//
// engine/model/attention.py:166-174 and :211-228 for a prefill: every prompt token
// attends to the keys of its own sequence at positions 0..pos (the causal mask of
// :219-222).  The reference runs one sequence per forward (execution_engine.py:85-111);
// here any number of sequences of any lengths go in one launch.  Rows
// [seq_start[s], seq_start[s+1]) are the tokens of sequence s, at positions
// seq_ctx0[s] + (row - seq_start[s]); their K/V are already in the pool, reached
// through block-table row s.
//
// A CTA owns one kv head and a tile of QT = 64 / REP consecutive tokens of one sequence.
// Its 64 MMA rows are the (token, query head) pairs of the tile that share the kv head
// (row m = token * REP + head), so each K/V block staged in shared memory serves QT
// tokens x REP heads, against REP heads of one token in the decode kernel.  The 4 warps
// (16 rows each) walk blocks 0..(last position of the tile) / 16 together through a
// kPfStages-deep cp.async ring; a warp skips the blocks that lie wholly after all of its
// rows.  Per row, online softmax in the log2 domain; a row's result depends only on its
// own keys and their block order, not on which other rows share its tile.
struct PrefillParams {
  const void* q;
  int64_t ld_q;
  int n_rows, nq, nkv;
  const void* k_cache;
  const void* v_cache;
  int64_t layer_off;  // elements
  int num_blocks;
  const int32_t* tables;
  int table_stride;
  const int32_t* seq_start;  // [n_seqs + 1], non-decreasing, within [0, n_rows]
  const int32_t* seq_ctx0;   // [n_seqs] keys already cached before the first row, or null (0)
  int n_seqs;
  float scale_log2;
  void* out;
  int64_t ld_out;
  int32_t* status;
};

constexpr int kPfWarps = 4;
constexpr int kPfRows = kPfWarps * 16;  // MMA rows per CTA
constexpr int kPfStages = 4;

template <int HD>
struct PfCfg {
  static constexpr size_t SMEM = (size_t)kPfStages * MmaCfg<HD>::STAGEB;
};

// Upper bound on the CTAs along x: sum_s ceil(len_s / QT) <= n_rows / QT + n_seqs.
static inline int prefill_tiles_bound(int n_rows, int n_seqs, int qt) { return n_rows / qt + n_seqs; }

template <int HD, int REP>
__global__ void __launch_bounds__(kPfWarps * 32) prefill_attn_mma_kernel(PrefillParams p) {
  pdl_wait();
  pdl_trigger();
  using C = MmaCfg<HD>;
  static_assert(kPfRows % REP == 0, "tile rows must hold whole tokens");
  constexpr int QT = kPfRows / REP;  // tokens per tile
  extern __shared__ __align__(128) uint8_t smem[];
  const int g = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int qr = lane >> 2, qt = lane & 3;

  // (sequence, tile) of this CTA.  Tiles are numbered sequence by sequence, each
  // sequence's last (longest) tile first; every warp finds the same answer.
  int seq = -1, tile = 0;
  {
    int base = 0;
    for (int s0 = 0; s0 < p.n_seqs && seq < 0; s0 += 32) {
      const int s = s0 + lane;
      int nt = 0;
      if (s < p.n_seqs) {
        const int len = p.seq_start[s + 1] - p.seq_start[s];
        nt = len > 0 ? (len + QT - 1) / QT : 0;
      }
      int inc = nt;  // inclusive prefix sum over the lanes
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
      }
      const int total = __shfl_sync(0xffffffffu, inc, 31);
      const int bx = (int)blockIdx.x - base;
      if (bx < total) {  // warp-uniform
        const unsigned hit = __ballot_sync(0xffffffffu, bx < inc);
        const int l = __ffs(hit) - 1;
        const int inc_l = __shfl_sync(0xffffffffu, inc, l);
        const int nt_l = __shfl_sync(0xffffffffu, nt, l);
        seq = s0 + l;
        tile = bx - (inc_l - nt_l);
      }
      base += total;
    }
  }
  if (seq < 0) return;  // past the last tile (the grid is an upper bound)
  const int rs = p.seq_start[seq], re = p.seq_start[seq + 1];
  const int ctx0 = p.seq_ctx0 ? p.seq_ctx0[seq] : 0;
  if (rs < 0 || re > p.n_rows || ctx0 < 0) {
    if (threadIdx.x == 0) raise_status(p.status, B2_DEV_RANGE);
    return;
  }
  const int len = re - rs;
  const int ntile = (len + QT - 1) / QT;
  const int t0 = (ntile - 1 - tile) * QT;  // first token of the tile within its sequence
  const int nt = min(QT, len - t0);        // tokens in the tile (>= 1)
  const int nblk = (ctx0 + t0 + nt - 1) / 16 + 1;
  const int32_t* table = p.tables + (int64_t)seq * p.table_stride;

  // This lane's two MMA rows (qr and qr + 8 of the warp's 16).
  const int m_lo = warp * 16 + qr, m_hi = m_lo + 8;
  const int tk_lo = m_lo / REP, tk_hi = m_hi / REP;
  const bool ok_lo = tk_lo < nt, ok_hi = tk_hi < nt;
  const int pos_lo = ctx0 + t0 + tk_lo, pos_hi = ctx0 + t0 + tk_hi;
  const int64_t row_lo = rs + t0 + tk_lo, row_hi = rs + t0 + tk_hi;
  const int col_lo = (g * REP + m_lo % REP) * HD, col_hi = (g * REP + m_hi % REP) * HD;
  // Last position any row of this warp attends to (warp-uniform).
  const int wpos = ctx0 + t0 + min(nt - 1, (warp * 16 + 15) / REP);

  // Q fragments: a0/a2 = row qr (k lo/hi), a1/a3 = row qr + 8.
  uint32_t qa[HD / 16][4];
  {
    const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(p.q);
    const __nv_bfloat16* qlo = ok_lo ? qb + row_lo * p.ld_q + col_lo : nullptr;
    const __nv_bfloat16* qhi = ok_hi ? qb + row_hi * p.ld_q + col_hi : nullptr;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      qa[kk][0] = ok_lo ? *reinterpret_cast<const uint32_t*>(qlo + kk * 16 + 2 * qt) : 0u;
      qa[kk][1] = ok_hi ? *reinterpret_cast<const uint32_t*>(qhi + kk * 16 + 2 * qt) : 0u;
      qa[kk][2] = ok_lo ? *reinterpret_cast<const uint32_t*>(qlo + kk * 16 + 8 + 2 * qt) : 0u;
      qa[kk][3] = ok_hi ? *reinterpret_cast<const uint32_t*>(qhi + kk * 16 + 8 + 2 * qt) : 0u;
    }
  }

  const int64_t tok_stride_b = (int64_t)p.nkv * HD * 2;
  const char* kbase = reinterpret_cast<const char*>(p.k_cache) + (p.layer_off + (int64_t)g * HD) * 2;
  const char* vbase = reinterpret_cast<const char*>(p.v_cache) + (p.layer_off + (int64_t)g * HD) * 2;
  const uint32_t sbase = smem_addr(smem);

  auto block_id = [&](int b) -> int { return b < p.table_stride ? table[b] : -1; };
  // All threads copy block b (K and V rows of this kv head) into ring slot b % kPfStages;
  // a block id outside the pool is not read, and the main loop skips that block.
  auto issue = [&](int b) {
    const int blk = block_id(b);
    if (blk < 0 || blk >= p.num_blocks) return;
    const uint32_t st = sbase + (uint32_t)((b % kPfStages) * C::STAGEB);
    const int64_t blk_off = (int64_t)blk * 16 * tok_stride_b;
    for (int i = threadIdx.x; i < 16 * C::CHUNKS; i += kPfWarps * 32) {
      const int r = i / C::CHUNKS, c = i % C::CHUNKS;
      const int64_t src = blk_off + r * tok_stride_b + c * 16;
      cp_async16(st + swz<HD>(r, c), kbase + src);
      cp_async16(st + C::BLKB + swz<HD>(r, c), vbase + src);
    }
  };

  float o[HD / 8][4];
#pragma unroll
  for (int d = 0; d < HD / 8; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  float m_lo_run = -INFINITY, m_hi_run = -INFINITY, l_lo = 0.f, l_hi = 0.f;

#pragma unroll
  for (int i = 0; i < kPfStages - 1; ++i) {
    if (i < nblk) issue(i);
    cp_async_commit();
  }
  for (int b = 0; b < nblk; ++b) {
    cp_async_wait<kPfStages - 2>();  // block b has landed (this thread's copies) ...
    __syncthreads();                 // ... for every thread, and slot (b - 1) is free
    if (b + kPfStages - 1 < nblk) issue(b + kPfStages - 1);
    cp_async_commit();
    const int blk = block_id(b);
    const bool blk_ok = blk >= 0 && blk < p.num_blocks;
    if (!blk_ok && threadIdx.x == 0) raise_status(p.status, B2_DEV_RANGE);
    // An out-of-range block was not copied (its ring slot is stale): skip it whole, like a
    // block whose every key follows every row of this warp.
    if (!blk_ok || b * 16 > wpos) continue;
    const uint32_t ks = sbase + (uint32_t)((b % kPfStages) * C::STAGEB);
    const uint32_t vs = ks + C::BLKB;

    // S = Q K^T over the block's 16 keys: two 8-key n-tiles.
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      const int mrow = (lane & 7) + ((lane >> 4) << 3);
      const int mchunk = kk * 2 + ((lane >> 3) & 1);
      uint32_t bf[4];
      ldsm_x4(ks + swz<HD>(mrow, mchunk), bf);
      mma_bf16(s[0], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], bf[0], bf[1]);
      mma_bf16(s[1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], bf[2], bf[3]);
    }
    // Scale, causal mask, online softmax for rows qr (elements 0, 1) and qr + 8 (2, 3).
    const int kb = b * 16;
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = kb + j * 8 + 2 * qt + e;
        const float vlo = (blk_ok && ok_lo && t <= pos_lo) ? s[j][e] * p.scale_log2 : -INFINITY;
        const float vhi = (blk_ok && ok_hi && t <= pos_hi) ? s[j][2 + e] * p.scale_log2 : -INFINITY;
        s[j][e] = vlo;
        s[j][2 + e] = vhi;
        mx_lo = fmaxf(mx_lo, vlo);
        mx_hi = fmaxf(mx_hi, vhi);
      }
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
    const float mn_lo = fmaxf(m_lo_run, mx_lo), mn_hi = fmaxf(m_hi_run, mx_hi);
    const float c_lo = safe_exp2_diff(m_lo_run, mn_lo), c_hi = safe_exp2_diff(m_hi_run, mn_hi);
    float pv[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        pv[j][e] = mn_lo == -INFINITY ? 0.f : safe_exp2_diff(s[j][e], mn_lo);
        pv[j][2 + e] = mn_hi == -INFINITY ? 0.f : safe_exp2_diff(s[j][2 + e], mn_hi);
      }
    l_lo = l_lo * c_lo + (pv[0][0] + pv[0][1] + pv[1][0] + pv[1][1]);
    l_hi = l_hi * c_hi + (pv[0][2] + pv[0][3] + pv[1][2] + pv[1][3]);
    m_lo_run = mn_lo;
    m_hi_run = mn_hi;
#pragma unroll
    for (int d = 0; d < HD / 8; ++d) {
      o[d][0] *= c_lo;
      o[d][1] *= c_lo;
      o[d][2] *= c_hi;
      o[d][3] *= c_hi;
    }
    // P (bf16) as the A operand: a0/a2 = row qr keys lo/hi, a1/a3 = row qr + 8.
    const uint32_t pa0 = pack_bf16(pv[0][0], pv[0][1]);
    const uint32_t pa1 = pack_bf16(pv[0][2], pv[0][3]);
    const uint32_t pa2 = pack_bf16(pv[1][0], pv[1][1]);
    const uint32_t pa3 = pack_bf16(pv[1][2], pv[1][3]);
#pragma unroll
    for (int d = 0; d < HD / 8; d += 2) {
      const int mrow = (lane & 7) + (((lane >> 3) & 1) << 3);
      const int mchunk = d + (lane >> 4);
      uint32_t bf[4];
      ldsm_x4_trans(vs + swz<HD>(mrow, mchunk), bf);
      mma_bf16(o[d], pa0, pa1, pa2, pa3, bf[0], bf[1]);
      mma_bf16(o[d + 1], pa0, pa1, pa2, pa3, bf[2], bf[3]);
    }
  }
  cp_async_wait<0>();
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(p.out);
  if (ok_lo) {
    __nv_bfloat16* dst = ob + row_lo * p.ld_out + col_lo + 2 * qt;
#pragma unroll
    for (int d = 0; d < HD / 8; ++d)
      *reinterpret_cast<uint32_t*>(dst + d * 8) =
          pack_bf16(l_lo > 0.f ? o[d][0] / l_lo : 0.f, l_lo > 0.f ? o[d][1] / l_lo : 0.f);
  }
  if (ok_hi) {
    __nv_bfloat16* dst = ob + row_hi * p.ld_out + col_hi + 2 * qt;
#pragma unroll
    for (int d = 0; d < HD / 8; ++d)
      *reinterpret_cast<uint32_t*>(dst + d * 8) =
          pack_bf16(l_hi > 0.f ? o[d][2] / l_hi : 0.f, l_hi > 0.f ? o[d][3] / l_hi : 0.f);
  }
}

// Opts a kernel into `bytes` of dynamic shared memory once per (kernel, device).
static int allow_dynamic_smem(const void* fn, size_t bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  B2_TRY_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({fn, dev})) return B2_OK;
  B2_TRY_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  done.insert({fn, dev});
  return B2_OK;
}

template <int HD, int W, int STAGES>
static int launch_mma_rep_cfg(int rep, const AttnParams& p, dim3 grid, cudaStream_t s) {
  const size_t smem = (size_t)W * STAGES * MmaCfg<HD>::STAGEB;
  auto go = [&](void (*k)(AttnParams)) -> int {
    const int rc = allow_dynamic_smem((const void*)k, smem);
    if (rc) return rc;
    B2_TRY_CUDA(launch_pdl(k, grid, dim3(W * 32), smem, s, p));
    return B2_OK;
  };
  switch (rep) {
    case 1: return go(paged_attn_mma_kernel<HD, 1, W, STAGES>);
    case 2: return go(paged_attn_mma_kernel<HD, 2, W, STAGES>);
    case 4: return go(paged_attn_mma_kernel<HD, 4, W, STAGES>);
    case 8: return go(paged_attn_mma_kernel<HD, 8, W, STAGES>);
    default: return fail(B2_ENOTSUP, "b2_paged_attention: nq/nkv = %d not supported (1, 2, 4, 8)", rep);
  }
}

// Grids of at most one CTA per SM (few (row, kv head, split) triples, e.g. one kv head
// per rank at TP=8) run 8 warps per CTA with 2-stage rings, so each SM still holds as
// many warps as two 4-warp CTAs.  The configuration follows from the grid alone, so two
// calls over the same shapes and split count (an eager call and a graph replay) give
// the same bits; between the two configurations only the float summation order differs.
template <int HD>
static int launch_mma_rep(int rep, const AttnParams& p, dim3 grid, cudaStream_t s) {
  const long ctas = (long)grid.x * grid.y * grid.z;
  if (ctas <= sm_count()) return launch_mma_rep_cfg<HD, 8, 2>(rep, p, grid, s);
  return launch_mma_rep_cfg<HD, kMmaWarps, kMmaStages>(rep, p, grid, s);
}

static int launch_mma(int hd, int rep, const AttnParams& p, dim3 grid, cudaStream_t s) {
  switch (hd) {
    case 32: return launch_mma_rep<32>(rep, p, grid, s);
    case 64: return launch_mma_rep<64>(rep, p, grid, s);
    case 128: return launch_mma_rep<128>(rep, p, grid, s);
    default: return fail(B2_ENOTSUP, "b2_paged_attention: bf16 head_dim %d not supported (32, 64, 128)", hd);
  }
}

template <int HD>
static int launch_prefill_rep(int rep, int n_rows, const PrefillParams& p, cudaStream_t s) {
  auto go = [&](void (*k)(PrefillParams), int qt) -> int {
    const int rc = allow_dynamic_smem((const void*)k, PfCfg<HD>::SMEM);
    if (rc) return rc;
    const dim3 grid(prefill_tiles_bound(n_rows, p.n_seqs, qt), p.nkv);
    B2_TRY_CUDA(launch_pdl(k, grid, dim3(kPfWarps * 32), PfCfg<HD>::SMEM, s, p));
    return B2_OK;
  };
  switch (rep) {
    case 1: return go(prefill_attn_mma_kernel<HD, 1>, kPfRows / 1);
    case 2: return go(prefill_attn_mma_kernel<HD, 2>, kPfRows / 2);
    case 4: return go(prefill_attn_mma_kernel<HD, 4>, kPfRows / 4);
    case 8: return go(prefill_attn_mma_kernel<HD, 8>, kPfRows / 8);
    default: return fail(B2_ENOTSUP, "b2_prefill_attention: nq/nkv = %d not supported (1, 2, 4, 8)", rep);
  }
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct AttnWs {
  size_t counters, ml, o, total;
};
// The counter region has a FIXED size so that calls with different row counts never
// read each other's partial states as counters.
constexpr size_t kAttnCounterSlots = 16384;

static AttnWs attn_ws_layout(int n_rows, int nq, int nkv, int hd, int splits) {
  AttnWs w{};
  if (splits <= 1) return w;
  w.counters = 0;
  w.ml = kAttnCounterSlots * sizeof(int);
  w.o = w.ml + align256((size_t)n_rows * nq * splits * 2 * sizeof(float));
  w.total = w.o + align256((size_t)n_rows * nq * splits * hd * sizeof(float));
  return w;
}

template <typename T, int HD>
static int launch_rep(int rep, const AttnParams& p, dim3 grid, cudaStream_t s) {
  auto go = [&](void (*k)(AttnParams)) -> int {
    B2_TRY_CUDA(launch_pdl(k, grid, dim3(kAttnWarps * 32), 0, s, p));
    return B2_OK;
  };
  switch (rep) {
    case 1: return go(paged_attn_simt_kernel<T, HD, 1>);
    case 2: return go(paged_attn_simt_kernel<T, HD, 2>);
    case 4: return go(paged_attn_simt_kernel<T, HD, 4>);
    case 8: return go(paged_attn_simt_kernel<T, HD, 8>);
    default: return fail(B2_ENOTSUP, "b2_paged_attention: nq/nkv = %d not supported (1, 2, 4, 8)", rep);
  }
}

template <typename T>
static int launch_hd(int hd, int rep, const AttnParams& p, dim3 grid, cudaStream_t s) {
  switch (hd) {
    case 32: return launch_rep<T, 32>(rep, p, grid, s);
    case 64: return launch_rep<T, 64>(rep, p, grid, s);
    case 128: return launch_rep<T, 128>(rep, p, grid, s);
    default: return fail(B2_ENOTSUP, "b2_paged_attention: head_dim %d not supported (32, 64, 128)", hd);
  }
}

// Scratch of b2_paged_attention_noalloc: a fixed array in the library's own device
// memory, present on every GPU that loads the library until the process exits.
constexpr size_t kNoAllocScratchBytes = (size_t)4 << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
constexpr int kNoAllocMaxDevices = 64;
static void* g_noalloc_scratch_addr[kNoAllocMaxDevices] = {nullptr};
static std::mutex g_noalloc_mutex;

// Device address of g_noalloc_scratch on the current device, looked up once per device.
// The name itself is only a host-side stand-in and must never reach a kernel.
static int noalloc_scratch(void** out) {
  int dev = 0;
  B2_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(B2_ENOTSUP, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(B2_ECUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev, cudaGetErrorString(e));
    g_noalloc_scratch_addr[dev] = p;
  }
  *out = g_noalloc_scratch_addr[dev];
  return B2_OK;
}

// Argument checks shared by b2_paged_attention and b2_paged_attention_noalloc (the
// latter runs them before it touches its shared scratch).  Workspace size is checked
// by the caller that owns the workspace.
static int check_paged_args(const void* q, int64_t ld_q, int n_rows, int nq, int nkv, int head_dim,
                            const void* k_cache, const void* v_cache, int layer, int num_blocks, int block_size,
                            const int32_t* block_tables, int table_stride, const int32_t* ctx_lens, void* out,
                            int64_t ld_out, int dtype, int num_splits) {
  B2_CHECK_ARG(n_rows >= 0 && nq > 0 && nkv > 0 && nq % nkv == 0, "b2_paged_attention: bad head counts");
  B2_CHECK_ARG(valid_dtype(dtype), "b2_paged_attention: bad dtype");
  B2_CHECK_ARG(num_blocks > 0 && block_size > 0 && table_stride > 0 && layer >= 0,
               "b2_paged_attention: bad cache geometry");
  B2_CHECK_ARG(num_splits >= 1 && num_splits <= 1024, "b2_paged_attention: num_splits %d out of [1, 1024]", num_splits);
  B2_CHECK_ARG(ld_q >= (int64_t)nq * head_dim && ld_out >= (int64_t)nq * head_dim,
               "b2_paged_attention: row strides too small");
  if (n_rows == 0) return B2_OK;
  B2_CHECK_ARG(q && k_cache && v_cache && block_tables && ctx_lens && out, "b2_paged_attention: null pointer");
  B2_CHECK_ARG(n_rows <= 65535, "b2_paged_attention: n_rows %d > 65535", n_rows);
  const size_t esz = dtype_bytes(dtype);
  B2_CHECK_ARG(((uintptr_t)q % 16) == 0 && ((ld_q * esz) % 16) == 0 && ((uintptr_t)k_cache % 16) == 0 &&
                   ((uintptr_t)v_cache % 16) == 0,
               "b2_paged_attention: q/cache must be 16-byte aligned");
  if (num_splits > 1)
    B2_CHECK_ARG((size_t)n_rows * nkv <= kAttnCounterSlots,
                 "b2_paged_attention: n_rows * nkv = %d exceeds %zu with num_splits > 1", n_rows * nkv,
                 kAttnCounterSlots);
  if (dtype == B2_BF16) B2_CHECK_ARG(block_size == 16, "b2_paged_attention: bf16 path needs block_size 16");
  return B2_OK;
}

}  // namespace b2

extern "C" {

size_t b2_paged_attention_workspace_bytes(int n_rows, int nq, int nkv, int head_dim, int num_splits) {
  return b2::attn_ws_layout(n_rows, nq, nkv, head_dim, num_splits).total;
}

int b2_paged_attention(const void* q, int64_t ld_q, int n_rows, int nq, int nkv, int head_dim,
                       const void* k_cache, const void* v_cache, int layer, int num_blocks,
                       int block_size, const int32_t* block_tables, int table_stride,
                       const int32_t* table_index, const int32_t* ctx_lens, int compat_pad,
                       float scale, void* out, int64_t ld_out, int dtype, void* workspace,
                       size_t workspace_bytes, int num_splits, int32_t* status, b2_stream_t stream) {
  const int rc = b2::check_paged_args(q, ld_q, n_rows, nq, nkv, head_dim, k_cache, v_cache, layer, num_blocks,
                                     block_size, block_tables, table_stride, ctx_lens, out, ld_out, dtype, num_splits);
  if (rc != B2_OK || n_rows == 0) return rc;
  b2::AttnWs lay = b2::attn_ws_layout(n_rows, nq, nkv, head_dim, num_splits);
  b2::AttnParams p{};
  if (num_splits > 1) {
    B2_CHECK_ARG(workspace && workspace_bytes >= lay.total,
                 "b2_paged_attention: workspace of %zu bytes needed, %zu given", lay.total, workspace_bytes);
    char* ws = static_cast<char*>(workspace);
    p.counters = reinterpret_cast<int*>(ws + lay.counters);
    p.ws_ml = reinterpret_cast<float*>(ws + lay.ml);
    p.ws_o = reinterpret_cast<float*>(ws + lay.o);
  }
  p.q = q;
  p.ld_q = ld_q;
  p.n_rows = n_rows;
  p.nq = nq;
  p.nkv = nkv;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.layer_off = (int64_t)layer * num_blocks * block_size * nkv * head_dim;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.tables = block_tables;
  p.table_stride = table_stride;
  p.table_index = table_index;
  p.ctx_lens = ctx_lens;
  p.compat_pad = compat_pad;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = out;
  p.ld_out = ld_out;
  p.splits = num_splits;
  p.status = status;
  dim3 grid(num_splits, nkv, n_rows);
  const int rep = nq / nkv;
  if (dtype == B2_BF16) return b2::launch_mma(head_dim, rep, p, grid, stream);
  return b2::launch_hd<float>(head_dim, rep, p, grid, stream);
}

// Same computation as b2_paged_attention, with the split scratch taken from the
// library's static device array instead of a caller-provided workspace.
int b2_paged_attention_noalloc(const void* q, int64_t ld_q, int n_rows, int nq, int nkv, int head_dim,
                               const void* k_cache, const void* v_cache, int layer, int num_blocks,
                               int block_size, const int32_t* block_tables, int table_stride,
                               const int32_t* table_index, const int32_t* ctx_lens, int compat_pad,
                               float scale, void* out, int64_t ld_out, int dtype, int num_splits,
                               int32_t* status, b2_stream_t stream) {
  // Every argument is checked before the shared scratch is touched: a rejected call must
  // not clear counters that a call still running on another stream is using.
  int rc = b2::check_paged_args(q, ld_q, n_rows, nq, nkv, head_dim, k_cache, v_cache, layer, num_blocks, block_size,
                                block_tables, table_stride, ctx_lens, out, ld_out, dtype, num_splits);
  if (rc != B2_OK || n_rows == 0) return rc;
  void* scratch = nullptr;
  if (num_splits > 1) {
    const size_t need = b2_paged_attention_workspace_bytes(n_rows, nq, nkv, head_dim, num_splits);
    B2_CHECK_ARG(need <= b2::kNoAllocScratchBytes,
                 "b2_paged_attention_noalloc: this call needs %zu bytes of split scratch but the static "
                 "array holds %zu; use fewer splits or rows, or b2_paged_attention with a workspace",
                 need, b2::kNoAllocScratchBytes);
    rc = b2::noalloc_scratch(&scratch);
    if (rc) return rc;
    // The array keeps the previous call's contents: zero the split counters this call uses.
    B2_TRY_CUDA(cudaMemsetAsync(scratch, 0, (size_t)n_rows * nkv * sizeof(int), stream));
  }
  return b2_paged_attention(q, ld_q, n_rows, nq, nkv, head_dim, k_cache, v_cache, layer, num_blocks, block_size,
                            block_tables, table_stride, table_index, ctx_lens, compat_pad, scale, out, ld_out,
                            dtype, scratch, scratch ? b2::kNoAllocScratchBytes : 0, num_splits, status, stream);
}


int b2_prefill_attention_tc(const void* q, int64_t ld_q, int n_rows, int nq, int nkv, int head_dim,
                            const void* k_cache, const void* v_cache, int layer, int num_blocks, int block_size,
                            const int32_t* block_tables, int table_stride, const int32_t* seq_start,
                            const int32_t* seq_ctx0, int n_seqs, float scale, void* out, int64_t ld_out, int dtype,
                            int32_t* status, b2_stream_t stream) {
  B2_CHECK_ARG(n_rows >= 0 && n_seqs >= 0 && nq > 0 && nkv > 0 && nq % nkv == 0,
               "b2_prefill_attention_tc: bad sizes");
  B2_CHECK_ARG(dtype == B2_BF16 && head_dim == 128 && block_size == 16,
               "b2_prefill_attention_tc: bf16, head_dim 128 and block_size 16 only");
  B2_CHECK_ARG(num_blocks > 0 && table_stride > 0 && layer >= 0, "b2_prefill_attention_tc: bad cache geometry");
  B2_CHECK_ARG(ld_q >= (int64_t)nq * head_dim && ld_out >= (int64_t)nq * head_dim,
               "b2_prefill_attention_tc: row strides too small");
  B2_CHECK_ARG(nkv <= 65535, "b2_prefill_attention_tc: nkv %d > 65535", nkv);
  if (n_rows == 0 || n_seqs == 0) return B2_OK;
  B2_CHECK_ARG(q && k_cache && v_cache && block_tables && seq_start && out && status,
               "b2_prefill_attention_tc: null pointer");
  const int64_t layer_off = (int64_t)layer * num_blocks * block_size * nkv * head_dim;
  return b2::prefill_attention_tc(q, ld_q, n_rows, nq, nkv, k_cache, v_cache, layer_off, num_blocks, block_tables,
                                  table_stride, seq_start, seq_ctx0, n_seqs, scale, out, ld_out, status, stream);
}

int b2_prefill_attention(const void* q, int64_t ld_q, int n_rows, int nq, int nkv, int head_dim,
                         const void* k_cache, const void* v_cache, int layer, int num_blocks, int block_size,
                         const int32_t* block_tables, int table_stride, const int32_t* seq_start,
                         const int32_t* seq_ctx0, int n_seqs, float scale, void* out, int64_t ld_out, int dtype,
                         int32_t* status, b2_stream_t stream) {
  B2_CHECK_ARG(n_rows >= 0 && n_seqs >= 0 && nq > 0 && nkv > 0 && nq % nkv == 0,
               "b2_prefill_attention: bad sizes");
  B2_CHECK_ARG(dtype == B2_BF16, "b2_prefill_attention: bf16 only (float32 prefill runs b2_paged_attention)");
  B2_CHECK_ARG(block_size == 16, "b2_prefill_attention: block_size %d (16 only)", block_size);
  B2_CHECK_ARG(num_blocks > 0 && table_stride > 0 && layer >= 0, "b2_prefill_attention: bad cache geometry");
  B2_CHECK_ARG(ld_q >= (int64_t)nq * head_dim && ld_out >= (int64_t)nq * head_dim,
               "b2_prefill_attention: row strides too small");
  B2_CHECK_ARG(nkv <= 65535, "b2_prefill_attention: nkv %d > 65535", nkv);
  if (n_rows == 0 || n_seqs == 0) return B2_OK;
  B2_CHECK_ARG(q && k_cache && v_cache && block_tables && seq_start && out && status,
               "b2_prefill_attention: null pointer");
  B2_CHECK_ARG(((uintptr_t)q % 4) == 0 && (ld_q % 2) == 0 && ((uintptr_t)out % 4) == 0 && (ld_out % 2) == 0 &&
                   ((uintptr_t)k_cache % 16) == 0 && ((uintptr_t)v_cache % 16) == 0,
               "b2_prefill_attention: q/out need 4-byte rows, the cache 16-byte alignment");
  if (head_dim == 128 && nkv <= 65535) {
    // the tensor-core kernel serves head_dim 128 with 16-byte aligned rows; anything it
    // declines (B2_ENOTSUP, nothing launched) runs on the mma.sync kernel below
    const int64_t layer_off = (int64_t)layer * num_blocks * block_size * nkv * head_dim;
    const int rc = b2::prefill_attention_tc(q, ld_q, n_rows, nq, nkv, k_cache, v_cache, layer_off, num_blocks,
                                            block_tables, table_stride, seq_start, seq_ctx0, n_seqs, scale, out,
                                            ld_out, status, stream);
    if (rc != B2_ENOTSUP) return rc;
  }
  b2::PrefillParams p{};
  p.q = q;
  p.ld_q = ld_q;
  p.n_rows = n_rows;
  p.nq = nq;
  p.nkv = nkv;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.layer_off = (int64_t)layer * num_blocks * block_size * nkv * head_dim;
  p.num_blocks = num_blocks;
  p.tables = block_tables;
  p.table_stride = table_stride;
  p.seq_start = seq_start;
  p.seq_ctx0 = seq_ctx0;
  p.n_seqs = n_seqs;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = out;
  p.ld_out = ld_out;
  p.status = status;
  const int rep = nq / nkv;
  switch (head_dim) {
    case 32: return b2::launch_prefill_rep<32>(rep, n_rows, p, stream);
    case 64: return b2::launch_prefill_rep<64>(rep, n_rows, p, stream);
    case 128: return b2::launch_prefill_rep<128>(rep, n_rows, p, stream);
    default: return b2::fail(B2_ENOTSUP, "b2_prefill_attention: head_dim %d not supported (32, 64, 128)", head_dim);
  }
}

}  // extern "C"
