// Causal varlen prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), head_dim 128.
//
// engine/model/attention.py:166-174 and :211-228 for a prefill: every prompt token attends
// to the keys of its own sequence at positions 0..pos (the causal mask of :219-222), for
// every prompt of a step in one launch (the reference runs one forward per prompt,
// execution_engine.py:85-111).  Rows [seq_start[s], seq_start[s+1]) are sequence s's
// tokens at positions seq_ctx0[s] + (row - seq_start[s]); their K/V are already in the
// paged pool (block-table row s).
//
// Work item = one kv head g and a tile of QT = 128 / REP consecutive tokens of one
// sequence: its 128 MMA rows are the (token, query head) pairs that share g, row
// m = token * REP + head, so every K/V tile serves QT tokens x REP heads.  The kernel is
// persistent (one CTA per SM walking items w = blockIdx.x, + gridDim.x, ...).  Per CTA:
//
//   warp 0 / lane 0 : TMA producer.  Q per item (a 3D box [QT tokens][REP heads][64 dims],
//                     twice for the two 64-dim halves, into one of two Q buffers, so the
//                     next item's Q loads during this one), then per KV tile of 64 keys the
//                     four 16-token pool blocks of K and of V (2D boxes [16 rows][64 dims]
//                     through the block table) into a 3-stage ring; 128-byte swizzle, no
//                     multicast.
//   warp 1 / lane 0 : MMA issuer.  S(j) = Q K(j)^T (M=128, N=64, K=128) into one of two
//                     TMEM S buffers; after S(j+1) is issued, PV(j) = P(j) V(j) (M=128,
//                     N=128, K=64; V read in place, MN-major) into one of two TMEM PV
//                     buffers.  tcgen05.commit signals each result and frees the K/V stage.
//   warps 2-9       : two threads per MMA row (TMEM lane): warps w and w + 4 share a lane
//                     quarter, each owning half of the row's 64 scores and 128 output dims.
//                     Softmax of S(j) in the log2 domain with the causal mask (the two
//                     halves exchange their row maxima through shared memory), P(j) to
//                     shared memory in bf16 (the A operand of PV(j)), then
//                     O = O * exp2(m_old - m_new) + PV(j-1) in registers; finally O / l.
//
// S(j+1) and PV(j-1) run on the tensor cores while the threads work on S(j).  Every wait
// is bounded by %globaltimer; a timeout raises B2_DEV_PIPE_TIMEOUT and the CTA drains its
// copies, frees TMEM and returns.  A block id outside the pool raises B2_DEV_RANGE and its
// keys are read from block 0 and masked (so no uninitialised shared memory is ever used).
#include <mutex>
#include <set>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace b2 {
namespace pftc {

using namespace b2::tc;

// Named barrier over the softmax warps only (the producer and MMA warps keep running).
__device__ __forceinline__ void softmax_sync() { asm volatile("bar.sync 1, %0;" ::"n"(32 * 8) : "memory"); }
// The same barrier, returning the AND of `pred` over all softmax threads, so that every
// softmax warp leaves the main loop in the same iteration (a warp waiting at a named
// barrier for a warp that already left would wait without bound).
__device__ __forceinline__ bool softmax_all(bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)pred), "n"(32 * 8)
      : "memory");
  return out != 0;
}

constexpr int HD = 128;
constexpr int ROWS = 128;                              // MMA M: (token, head) rows per CTA
constexpr int KT = 64;                                 // keys per KV tile (4 pool blocks)
constexpr int ST = 3;                                  // KV ring stages
constexpr int kSoftWarps = 8;                          // two per TMEM lane quarter: each owns half a row
constexpr int kThreads = 64 + 32 * kSoftWarps;         // producer, MMA, softmax warps
constexpr uint32_t HALF = KT * 64 * 2;                 // 8 KB: 64 keys x 64 dims
constexpr uint32_t STAGE = 4 * HALF;                   // K lo | K hi | V lo | V hi
constexpr uint32_t P_BYTES = ROWS * KT * 2;            // 16 KB
constexpr uint32_t Q_HALF = ROWS * 64 * 2;             // 16 KB
// Layout (1024-byte aligned): the K/V ring first, then P[2], then Q[2] (lo | hi each).
constexpr uint32_t OFF_P = ST * STAGE;
constexpr uint32_t OFF_Q = OFF_P + 2 * P_BYTES;
constexpr size_t SMEM = OFF_Q + 4 * Q_HALF + 1024;
constexpr uint32_t TMEM_COLS = 512;                    // S[2] (64 each) + PV[2] (128 each), rounded up
constexpr uint32_t COL_S = 0, COL_PV = 128;

struct Params {
  int n_rows, nq, nkv;
  int num_blocks;
  const int32_t* tables;
  int table_stride;
  const int32_t* seq_start;
  const int32_t* seq_ctx0;
  int n_seqs;
  float scale_log2;
  void* out;
  int64_t ld_out;
  int32_t* status;
};

// Shared-memory descriptor of an MN-major operand with 128-byte swizzle: 64-element rows
// along N (128 bytes), 8-row groups along K `sbo` bytes apart, the next 64 N-elements
// `lbo` bytes on (sm_100 descriptor version 1).
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// One work item: a tile of QT tokens of one sequence, for one kv head.
struct Item {
  int rs, t0, nt, ctx0, n_kv, g;
  const int32_t* table;
  bool valid;
};

// Tiles of QT tokens over all sequences (every lane of the calling warp gets the total).
__device__ __forceinline__ int count_tiles(const Params& p, int qt, int lane) {
  int total = 0;
  for (int s0 = 0; s0 < p.n_seqs; s0 += 32) {
    const int s = s0 + lane;
    int nt = 0;
    if (s < p.n_seqs) {
      const int len = p.seq_start[s + 1] - p.seq_start[s];
      nt = len > 0 ? (len + qt - 1) / qt : 0;
    }
    total += __reduce_add_sync(0xffffffffu, nt);
  }
  return total;
}

// Item w: kv head w % nkv of tile w / nkv, tiles numbered sequence by sequence with each
// sequence's last (longest) tile first.  Every warp computes the same answer (warp prefix
// sums over the sequences); all lanes of the calling warp take part.
template <int QT>
__device__ Item find_item(const Params& p, int w, int lane) {
  Item it{};
  it.valid = false;
  const int bx = w / p.nkv;
  it.g = w % p.nkv;
  int seq = -1, tile = 0, base = 0;
  for (int s0 = 0; s0 < p.n_seqs && seq < 0; s0 += 32) {
    const int s = s0 + lane;
    int nt = 0;
    if (s < p.n_seqs) {
      const int len = p.seq_start[s + 1] - p.seq_start[s];
      nt = len > 0 ? (len + QT - 1) / QT : 0;
    }
    int inc = nt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += v;
    }
    const int total = __shfl_sync(0xffffffffu, inc, 31);
    const int b = bx - base;
    if (b < total) {
      const unsigned hit = __ballot_sync(0xffffffffu, b < inc);
      const int l = __ffs(hit) - 1;
      const int inc_l = __shfl_sync(0xffffffffu, inc, l);
      const int nt_l = __shfl_sync(0xffffffffu, nt, l);
      seq = s0 + l;
      tile = b - (inc_l - nt_l);
    }
    base += total;
  }
  if (seq < 0) return it;
  const int rs = p.seq_start[seq], re = p.seq_start[seq + 1];
  const int ctx0 = p.seq_ctx0 ? p.seq_ctx0[seq] : 0;
  if (rs < 0 || re > p.n_rows || ctx0 < 0) {
    if (lane == 0) raise_status(p.status, B2_DEV_RANGE);
    return it;
  }
  const int len = re - rs;
  const int ntile = (len + QT - 1) / QT;
  it.rs = rs;
  it.t0 = (ntile - 1 - tile) * QT;  // first token of the tile within its sequence
  it.nt = min(QT, len - it.t0);     // tokens in the tile (>= 1)
  it.ctx0 = ctx0;
  it.n_kv = (ctx0 + it.t0 + it.nt - 1) / KT + 1;  // KV tiles of 64 keys up to the last position
  it.table = p.tables + (int64_t)seq * p.table_stride;
  it.valid = true;
  return it;
}

// Persistent: one CTA per SM walks the items w = blockIdx.x, + gridDim.x, ...; barriers,
// TMEM and the rings are set up once, the producer prefetches the next item's Q into the
// second Q buffer, and tile counters (ring stages, S/PV buffers, barrier phases) run on
// across items.
template <int REP>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const Params p) {
  constexpr int QT = ROWS / REP;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full[2];
  __shared__ __align__(8) uint64_t q_empty[2];
  __shared__ __align__(8) uint64_t kv_full[ST];
  __shared__ __align__(8) uint64_t kv_empty[ST];
  __shared__ __align__(8) uint64_t s_full[2];
  __shared__ __align__(8) uint64_t s_empty[2];
  __shared__ __align__(8) uint64_t p_full[2];
  __shared__ __align__(8) uint64_t pv_full[2];
  __shared__ __align__(8) uint64_t pv_empty[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ float s_red[2][2][ROWS];  // [tile parity][half][row]: the halves' row maxima
  __shared__ float s_l[2][ROWS];       // [half][row]: the halves' final sums of probabilities

  pdl_wait();  // the metadata, q and the pool may come from the preceding kernels
  pdl_trigger();
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = count_tiles(p, QT, lane) * p.nkv;
  if ((int)blockIdx.x >= n_items) return;  // nothing allocated yet

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 1);
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], kSoftWarps);
      mbar_init(&p_full[b], kSoftWarps);
      mbar_init(&pv_full[b], 1);
      mbar_init(&pv_empty[b], kSoftWarps);
    }
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer
    const uint64_t pol_q = policy_evict_first();
    const uint64_t pol_kv = policy_evict_last();  // K/V tiles are re-read by the sequence's other tiles
    int i = 0, J = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
      const Item it = find_item<QT>(p, w, lane);
      if (!it.valid) continue;
      if (lane == 0) {
        const int qb = i & 1;
        if (!mbar_wait(&q_empty[qb], ((uint32_t)(i >> 1) & 1u) ^ 1u)) {
          raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
          ok = false;
        } else {
          uint8_t* qs = smem + OFF_Q + qb * 2 * Q_HALF;
          mbar_arrive_expect_tx(&q_full[qb], 2 * Q_HALF);
          tma_load_3d(qs, &tmQ, &q_full[qb], 0, it.g * REP, it.rs + it.t0, pol_q);
          tma_load_3d(qs + Q_HALF, &tmQ, &q_full[qb], 64, it.g * REP, it.rs + it.t0, pol_q);
        }
        const int last_pos = it.ctx0 + it.t0 + it.nt - 1;
        for (int j = 0; j < it.n_kv && ok; ++j, ++J) {
          const int st = J % ST;
          if (!mbar_wait(&kv_empty[st], ((uint32_t)(J / ST) & 1u) ^ 1u)) {
            raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
            ok = false;
            break;
          }
          uint8_t* sb = smem + (size_t)st * STAGE;
          mbar_arrive_expect_tx(&kv_full[st], STAGE);
          for (int b = 0; b < KT / 16; ++b) {
            const int bi = j * (KT / 16) + b;
            int blk = bi < p.table_stride ? it.table[bi] : -1;
            if (blk < 0 || blk >= p.num_blocks) {
              // A block holding keys some row attends to must exist; past the last position
              // the keys are masked and any valid block serves as filler.
              if (bi * 16 <= last_pos) raise_status(p.status, B2_DEV_RANGE);
              blk = 0;
            }
            const int y = blk * 16;
            tma_load_2d(sb + b * 2048, &tmK, &kv_full[st], it.g * HD, y, pol_kv);
            tma_load_2d(sb + HALF + b * 2048, &tmK, &kv_full[st], it.g * HD + 64, y, pol_kv);
            tma_load_2d(sb + 2 * HALF + b * 2048, &tmV, &kv_full[st], it.g * HD, y, pol_kv);
            tma_load_2d(sb + 3 * HALF + b * 2048, &tmV, &kv_full[st], it.g * HD + 64, y, pol_kv);
          }
        }
      }
      ++i;
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (lane == 0) {
      // Copies still in flight (only after an aborted pipeline) land before the CTA exits.
      for (int q = 0; q < 2 && q < i; ++q) {
        const int last_q = q + ((i - 1 - q) / 2) * 2;
        mbar_wait(&q_full[q], (uint32_t)(last_q >> 1) & 1u, 100000000ull);
      }
      for (int st = 0; st < ST && st < J; ++st) {
        const int last_i = st + ((J - 1 - st) / ST) * ST;
        mbar_wait(&kv_full[st], (uint32_t)(last_i / ST) & 1u, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc_s = instr_desc_bf16(ROWS, KT);
    constexpr uint32_t idesc_pv = instr_desc_bf16(ROWS, HD) | (1u << 16);  // B (V) MN-major
    int i = 0, J = 0;
    bool ok = true;
    auto issue_pv = [&](int Jx) -> bool {  // PV of global tile Jx
      const int b = Jx & 1;
      if (!mbar_wait(&p_full[b], (uint32_t)(Jx >> 1) & 1u) ||
          !mbar_wait(&pv_empty[b], ((uint32_t)(Jx >> 1) & 1u) ^ 1u)) {
        raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
        return false;
      }
      tc_fence_after();
      const uint32_t p_addr = smem_u32(smem + OFF_P + b * P_BYTES);
      const uint32_t v_addr = smem_u32(smem + (size_t)(Jx % ST) * STAGE + 2 * HALF);
#pragma unroll
      for (int kk = 0; kk < KT / 16; ++kk)  // 16 keys per MMA: +32 bytes of P rows, +2 KB of V rows
        umma_bf16(tmem + COL_PV + b * HD, smem_desc_sw128(p_addr) + 2 * kk,
                  smem_desc_sw128_mn(v_addr + kk * 2048, HALF, 1024), idesc_pv, kk > 0 ? 1u : 0u);
      umma_commit(&pv_full[b]);
      umma_commit(&kv_empty[Jx % ST]);
      return true;
    };
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
      const Item it = find_item<QT>(p, w, lane);
      if (!it.valid) continue;
      if (lane == 0) {
        const int qb = i & 1;
        if (!mbar_wait(&q_full[qb], (uint32_t)(i >> 1) & 1u)) {
          raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
          ok = false;
        }
        const uint32_t q_addr = smem_u32(smem + OFF_Q + qb * 2 * Q_HALF);
        for (int j = 0; j < it.n_kv && ok; ++j, ++J) {
          const int st = J % ST, b = J & 1;
          if (!mbar_wait(&kv_full[st], (uint32_t)(J / ST) & 1u) ||
              !mbar_wait(&s_empty[b], ((uint32_t)(J >> 1) & 1u) ^ 1u)) {
            raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + (size_t)st * STAGE);
#pragma unroll
          for (int half = 0; half < 2; ++half)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16(tmem + COL_S + b * KT, smem_desc_sw128(q_addr + half * Q_HALF) + 2 * kk,
                        smem_desc_sw128(k_addr + half * HALF) + 2 * kk, idesc_s, (half | kk) ? 1u : 0u);
          umma_commit(&s_full[b]);
          if (j >= 1 && !issue_pv(J - 1)) {
            ok = false;
            break;
          }
        }
        if (ok) ok = issue_pv(J - 1);  // the item's last tile
        umma_commit(&q_empty[qb]);     // every S MMA of this item has read Q buffer qb
      }
      ++i;
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (lane == 0) {
      umma_commit(&drain_bar);  // every MMA issued by this thread has completed once it fires
      mbar_wait(&drain_bar, 0, 100000000ull);
    }
    __syncwarp();
  } else {
    // ---------------- softmax / accumulation: two threads per MMA row
    const int sw = warp - 2;                 // 0..7
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int half = sw >> 2;                // which half of the row's scores and dims
    const int m = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int tk = m / REP, h = m % REP;
    int J = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
      const Item it = find_item<QT>(p, w, lane);
      if (!it.valid) continue;
      const bool row_ok = tk < it.nt;
      const int pos = it.ctx0 + it.t0 + tk;  // this row's token position (the last key it attends to)
      float o[HD / 2];
#pragma unroll
      for (int c = 0; c < HD / 2; ++c) o[c] = 0.f;
      float m_run = -INFINITY, l_run = 0.f, m_o = -INFINITY;
      float m_tile[2] = {-INFINITY, -INFINITY};
      auto accumulate = [&](int Jx) {  // O = O * exp2(m_o - m(Jx)) + PV(Jx), this thread's 64 dims
        const int b = Jx & 1;
        // warp-uniform verdict: the TMEM loads below are .sync.aligned
        const bool done = __all_sync(0xffffffffu, mbar_wait(&pv_full[b], (uint32_t)(Jx >> 1) & 1u));
        if (!done) {
          if (lane == 0) raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
          ok = false;
        }
        tc_fence_after();
        uint32_t r0[32], r1[32];
        const uint32_t a = tmem + lane_off + COL_PV + b * HD + half * (HD / 2);
        tmem_ld32_nowait(a, r0);
        tmem_ld32_nowait(a + 32, r1);
        tmem_wait_ld();
        const float mi = m_tile[b];
        const float corr = (m_o == -INFINITY) ? 0.f : exp2f(m_o - mi);
        if (done) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            o[e] = o[e] * corr + __uint_as_float(r0[e]);
            o[32 + e] = o[32 + e] * corr + __uint_as_float(r1[e]);
          }
          m_o = mi;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pv_empty[b]);
      };
      for (int j = 0; j < it.n_kv; ++j, ++J) {
        const int b = J & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (uint32_t)(J >> 1) & 1u))) {
          if (lane == 0) raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
          ok = false;
        }
        // both halves of every row meet at the exchange below, so a failed wait still runs
        // the barrier (with nothing valid) before every softmax warp leaves the loop
        tc_fence_after();
        uint32_t sr[32];
        tmem_ld32_nowait(tmem + lane_off + COL_S + b * KT + half * 32, sr);
        tmem_wait_ld();
        const int k0 = j * KT + half * 32;
        float sv[32];
        float mx = -INFINITY;
        if (ok && row_ok && k0 + 31 <= pos) {  // every key of this half-tile is visible (the common case)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            sv[e] = __uint_as_float(sr[e]) * p.scale_log2;
            mx = fmaxf(mx, sv[e]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const bool valid = ok && row_ok && k0 + e <= pos;
            sv[e] = valid ? __uint_as_float(sr[e]) * p.scale_log2 : -INFINITY;
            mx = fmaxf(mx, sv[e]);
          }
        }
        s_red[J & 1][half][m] = mx;
        ok = softmax_all(ok);
        mx = fmaxf(mx, s_red[J & 1][half ^ 1][m]);
        if (!ok) break;
        const float m_new = fmaxf(m_run, mx);
        // P = exp2(s - m_new) in bf16 into this half's four 16-byte chunks of the swizzled row
        uint8_t* prow = smem + OFF_P + b * P_BYTES + m * 128;
        float lsum = 0.f;
        // a row with nothing visible yet keeps p = 0 (exp2(-inf - -inf) would be NaN)
        const float m_sub = m_new == -INFINITY ? 0.f : m_new;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t wv[4];
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const int e = q * 8 + e2 * 2;
            const float p0 = exp2f(sv[e] - m_sub);  // sv = -inf (masked) gives 0
            const float p1 = exp2f(sv[e + 1] - m_sub);
            lsum += p0 + p1;
            __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
            wv[e2] = *reinterpret_cast<uint32_t*>(&h2);
          }
          const int chunk = half * 4 + q;
          *reinterpret_cast<uint4*>(prow + ((chunk ^ (m & 7)) << 4)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
        l_run = (m_run == -INFINITY ? 0.f : l_run * exp2f(m_run - m_new)) + lsum;
        m_run = m_new;
        m_tile[b] = m_new;
        fence_proxy_async_smem();  // P[b] written by these threads is read by the tensor cores
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s_empty[b]);
          mbar_arrive(&p_full[b]);
        }
        if (j >= 1) accumulate(J - 1);
      }
      // No early exit here: a failed wait inside accumulate() is per warp, and every softmax
      // warp must reach the exchange below, which makes the verdict uniform again.
      if (ok) accumulate(J - 1);  // the item's last tile
      // the row's sum of probabilities is the sum of the two halves' (same running maximum)
      s_l[half][m] = l_run;
      ok = softmax_all(ok);
      const float l_tot = l_run + s_l[half ^ 1][m];
      // O / l to global memory: this thread's 64 dims of the row, 16-byte stores
      if (ok && row_ok) {
        const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)(it.rs + it.t0 + tk) * p.ld_out +
                             (int64_t)(it.g * REP + h) * HD + half * (HD / 2);
#pragma unroll
        for (int c = 0; c < HD / 2; c += 8) {
          uint32_t wv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            __nv_bfloat162 h2 = __floats2bfloat162_rn(o[c + 2 * u] * inv, o[c + 2 * u + 1] * inv);
            wv[u] = *reinterpret_cast<uint32_t*>(&h2);
          }
          *reinterpret_cast<uint4*>(dst + c) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
      }
    }
  }

  // ---------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

static int allow_smem_once(const void* fn, size_t bytes) {
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

static int encode(CUtensorMap* m, const void* ptr, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                  const cuuint32_t* box) {
  auto fn = encode_fn();
  if (!fn) return fail(B2_ECUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B2_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return B2_OK;
}

}  // namespace pftc

// Launches the tensor-core prefill attention (bf16, head_dim 128).  Returns B2_ENOTSUP,
// launching nothing, for shapes it does not serve.
int prefill_attention_tc(const void* q, int64_t ld_q, int n_rows, int nq, int nkv, const void* k_cache,
                         const void* v_cache, int64_t layer_off, int num_blocks, const int32_t* tables,
                         int table_stride, const int32_t* seq_start, const int32_t* seq_ctx0, int n_seqs,
                         float scale, void* out, int64_t ld_out, int32_t* status, cudaStream_t stream) {
  using namespace pftc;
  const int rep = nq / nkv;
  if (!(rep == 1 || rep == 2 || rep == 4 || rep == 8)) return fail(B2_ENOTSUP, "prefill tc: nq/nkv = %d", rep);
  if (((uintptr_t)q % 16) || (ld_q % 8) || ((uintptr_t)k_cache % 16) || ((uintptr_t)v_cache % 16) ||
      ((uintptr_t)out % 16) || (ld_out % 8))
    return fail(B2_ENOTSUP, "prefill tc: q/out rows and the pool need 16-byte alignment");
  Params p{};
  p.n_rows = n_rows;
  p.nq = nq;
  p.nkv = nkv;
  p.num_blocks = num_blocks;
  p.tables = tables;
  p.table_stride = table_stride;
  p.seq_start = seq_start;
  p.seq_ctx0 = seq_ctx0;
  p.n_seqs = n_seqs;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = out;
  p.ld_out = ld_out;
  p.status = status;
  const int qt = ROWS / rep;
  CUtensorMap mq, mk, mv;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)nq, (cuuint64_t)n_rows};
    const cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)ld_q * 2};
    const cuuint32_t box[3] = {64, (cuuint32_t)rep, (cuuint32_t)qt};
    const int rc = encode(&mq, q, 3, dims, strides, box);
    if (rc) return rc;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)nkv * HD, (cuuint64_t)num_blocks * 16};
    const cuuint64_t strides[1] = {(cuuint64_t)nkv * HD * 2};
    const cuuint32_t box[2] = {64, 16};
    const char* kb = static_cast<const char*>(k_cache) + layer_off * 2;
    const char* vb = static_cast<const char*>(v_cache) + layer_off * 2;
    int rc = encode(&mk, kb, 2, dims, strides, box);
    if (rc) return rc;
    rc = encode(&mv, vb, 2, dims, strides, box);
    if (rc) return rc;
  }
  const long items = (long)(n_rows / qt + n_seqs) * nkv;  // an upper bound; the kernel counts exactly
  const dim3 grid((unsigned)(items < sm_count() ? items : sm_count()));
  auto go = [&](void (*k)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const Params)) -> int {
    const int rc = allow_smem_once((const void*)k, SMEM);
    if (rc) return rc;
    B2_TRY_CUDA(launch_pdl(k, grid, dim3(kThreads), SMEM, stream, mq, mk, mv, p));
    return B2_OK;
  };
  switch (rep) {
    case 1: return go(prefill_attn_tc_kernel<1>);
    case 2: return go(prefill_attn_tc_kernel<2>);
    case 4: return go(prefill_attn_tc_kernel<4>);
    default: return go(prefill_attn_tc_kernel<8>);
  }
}

}  // namespace b2
