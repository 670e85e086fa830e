// Causal varlen prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), head_dim 128.
//
// engine/model/attention.py:166-174 and :211-228 for a prefill: every prompt token attends
// to the keys of its own sequence at positions 0..pos (the causal mask of :219-222), for
// every prompt of a step in one launch (the reference runs one forward per prompt,
// execution_engine.py:85-111).  Rows [seq_start[s], seq_start[s+1]) are sequence s's
// tokens at positions seq_ctx0[s] + (row - seq_start[s]); their K/V are already in the
// paged pool (block-table row s).
//
// A Q tile is QT = 128 / REP consecutive tokens of one sequence for one kv head g: its 128
// MMA rows are the (token, query head) pairs that share g, row m = token * REP + head, so
// every K/V tile serves QT tokens x REP heads.  Work item = one kv head and a PAIR of
// adjacent Q tiles of one sequence (the later tile in group 0, the one before it in group
// 1), which read the same K/V tiles: each K/V tile brought into shared memory feeds two
// S = Q K^T products.  The kernel is persistent (one CTA per SM walking items w =
// blockIdx.x, + gridDim.x, ...).  Per CTA:
//
//   warp 0 / lane 0 : TMA producer.  Per item the two Q tiles (3D boxes [QT tokens][REP
//                     heads][64 dims], two per tile for the 64-dim halves), then per K/V
//                     tile of 64 keys the four 16-token pool blocks of K and of V (2D boxes
//                     [16 rows][64 dims] through the block table) into a 3-stage ring;
//                     128-byte swizzle, no multicast.
//   warp 1 / lane 0 : MMA issuer.  Per K/V tile j: S_g(j) = Q_g K(j)^T (M=128, N=64, K=128)
//                     for both groups into one of each group's two TMEM S buffers, then
//                     O_g += P_g(j-1) V(j-1) (M=128, N=128, K=64; P read from TMEM, V in
//                     place from shared memory as an MN-major operand) into each group's
//                     TMEM O accumulator.
//   warps 2-5, 6-9  : softmax of group 0 and group 1, one thread per MMA row (TMEM lane):
//                     the row's 64 scores of S(j) with the causal mask in the log2 domain,
//                     P(j) in bf16 back into TMEM over the S(j) it was computed from (the A
//                     operand of PV(j)), the running sum of probabilities; at the end O / l.
//
// O stays in TMEM.  P(j) is taken relative to the row's reference maximum m_ref, which
// moves only when a tile's maximum exceeds it by more than 8 (a factor of 256): then the
// warp rescales its rows of O in TMEM (after PV(j-1) has completed) and the running sum.
// exp2(s - m_ref) <= 256 keeps P exact to bf16 and O, l in float32 range, and O / l does
// not depend on the reference chosen, so the result is the softmax of the reference's
// formula.  No barrier couples the warps: every hand-off is an mbarrier, tested a step
// ahead where the answer would otherwise stall the tensor cores, and every wait is bounded
// by %globaltimer; a timeout raises B2_DEV_PIPE_TIMEOUT and the CTA drains its
// copies, frees TMEM and returns.  A block id outside the pool raises B2_DEV_RANGE and its
// keys are read from block 0 and masked (so no uninitialised shared memory is ever used).
#include <mutex>
#include <set>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace b2 {
namespace pftc {

using namespace b2::tc;

constexpr int HD = 128;
constexpr int ROWS = 128;                              // MMA M: (token, head) rows per Q tile
constexpr int KT = 64;                                 // keys per KV tile (4 pool blocks)
constexpr int ST = 3;                                  // KV ring stages
constexpr int NG = 2;                                  // Q tiles (softmax groups) per item
constexpr int kGroupWarps = 4;                         // one per TMEM lane quarter
constexpr int kThreads = 64 + 32 * NG * kGroupWarps;   // producer, MMA, softmax warps
constexpr uint32_t HALF = KT * 64 * 2;                 // 8 KB: 64 keys x 64 dims
constexpr uint32_t STAGE = 4 * HALF;                   // K lo | K hi | V lo | V hi
constexpr uint32_t Q_HALF = ROWS * 64 * 2;             // 16 KB
constexpr uint32_t Q_BYTES = 2 * Q_HALF;               // one Q tile, lo | hi
// Layout (1024-byte aligned): the K/V ring, then Q[NG][2] (the next item's Q tiles load
// while this item runs): 225 KB.
constexpr uint32_t OFF_Q = ST * STAGE;
constexpr size_t SMEM = OFF_Q + NG * 2 * Q_BYTES + 1024;
static_assert(SMEM + 512 <= 232448, "shared memory above the 227 KB a CTA may use");
// TMEM per group (256 columns): S[2] (64 each) then O (128); 512 in all.  P(j) in bf16
// overwrites the first 32 columns of S(j)'s buffer once the softmax has read S(j).
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t GROUP_COLS = 256, COL_S = 0, COL_O = 128;
constexpr float kRescale = 8.f;                        // log2 of the largest P before O is rescaled

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

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 32 lanes x 32 consecutive 32-bit columns stored to TMEM (the caller waits with
// tmem_wait_st() before the tensor cores may read them).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// One work item: kv head g and up to two Q tiles of one sequence (tile 1 may be empty).
struct Item {
  int rs, ctx0, g;
  int t0[NG], nt[NG], n_kv[NG];
  const int32_t* table;
  bool valid;
};

// Q-tile pairs of QT tokens over all sequences (every lane of the calling warp gets the total).
__device__ __forceinline__ int count_pairs(const Params& p, int qt, int lane) {
  int total = 0;
  for (int s0 = 0; s0 < p.n_seqs; s0 += 32) {
    const int s = s0 + lane;
    int np = 0;
    if (s < p.n_seqs) {
      const int len = p.seq_start[s + 1] - p.seq_start[s];
      np = len > 0 ? ((len + qt - 1) / qt + 1) / 2 : 0;
    }
    total += __reduce_add_sync(0xffffffffu, np);
  }
  return total;
}

// Item w: kv head w % nkv of pair w / nkv, pairs numbered sequence by sequence with each
// sequence's last (longest) tiles first: pair u holds tiles 2u and 2u + 1 counted from the
// end of the sequence.  Every warp computes the same answer (warp prefix sums over the
// sequences); all lanes of the calling warp take part.
template <int QT>
__device__ Item find_item(const Params& p, int w, int lane) {
  Item it{};
  it.valid = false;
  const int bx = w / p.nkv;
  it.g = w % p.nkv;
  int seq = -1, pair = 0, base = 0;
  for (int s0 = 0; s0 < p.n_seqs && seq < 0; s0 += 32) {
    const int s = s0 + lane;
    int np = 0;
    if (s < p.n_seqs) {
      const int len = p.seq_start[s + 1] - p.seq_start[s];
      np = len > 0 ? ((len + QT - 1) / QT + 1) / 2 : 0;
    }
    int inc = np;
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
      const int np_l = __shfl_sync(0xffffffffu, np, l);
      seq = s0 + l;
      pair = b - (inc_l - np_l);
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
#pragma unroll
  for (int q = 0; q < NG; ++q) {
    const int tile = 2 * pair + q;  // counted from the end of the sequence
    if (tile < ntile) {
      it.t0[q] = (ntile - 1 - tile) * QT;          // first token of the tile within its sequence
      it.nt[q] = min(QT, len - it.t0[q]);          // tokens in the tile (>= 1)
      it.n_kv[q] = (ctx0 + it.t0[q] + it.nt[q] - 1) / KT + 1;  // KV tiles up to its last position
    } else {
      it.t0[q] = 0;
      it.nt[q] = 0;
      it.n_kv[q] = 0;
    }
  }
  it.rs = rs;
  it.ctx0 = ctx0;
  it.table = p.tables + (int64_t)seq * p.table_stride;
  it.valid = true;
  return it;
}

template <int REP>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const Params p) {
  constexpr int QT = ROWS / REP;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full[NG][2];
  __shared__ __align__(8) uint64_t q_empty[NG][2];
  __shared__ __align__(8) uint64_t kv_full[ST];
  __shared__ __align__(8) uint64_t kv_empty[ST];
  __shared__ __align__(8) uint64_t s_full[NG][2];
  __shared__ __align__(8) uint64_t p_full[NG][2];
  __shared__ __align__(8) uint64_t pv_done[NG][2];
  __shared__ __align__(8) uint64_t o_empty[NG];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;

  pdl_wait();  // the metadata, q and the pool may come from the preceding kernels
  pdl_trigger();
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = count_pairs(p, QT, lane) * p.nkv;
  if ((int)blockIdx.x >= n_items) return;  // nothing allocated yet

  if (threadIdx.x == 0) {
    for (int g = 0; g < NG; ++g) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&q_full[g][b], 1);
        mbar_init(&q_empty[g][b], 1);
      }
      for (int b = 0; b < 2; ++b) mbar_init(&s_full[g][b], 1);
      for (int b = 0; b < 2; ++b) {
        mbar_init(&p_full[g][b], kGroupWarps);
        mbar_init(&pv_done[g][b], 1);
      }
      mbar_init(&o_empty[g], kGroupWarps);
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
    int iq[NG] = {0, 0};  // Q loads into each group's buffer
    int J = 0;            // K/V tiles through the ring
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
      const Item it = find_item<QT>(p, w, lane);
      if (!it.valid) continue;
      if (lane == 0) {
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          if (it.nt[g] == 0 || !ok) continue;
          const int qb = iq[g] & 1;
          if (!mbar_wait(&q_empty[g][qb], ((uint32_t)(iq[g] >> 1) & 1u) ^ 1u)) {
            raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
            ok = false;
            continue;
          }
          uint8_t* qs = smem + OFF_Q + (g * 2 + qb) * Q_BYTES;
          mbar_arrive_expect_tx(&q_full[g][qb], Q_BYTES);
          tma_load_3d(qs, &tmQ, &q_full[g][qb], 0, it.g * REP, it.rs + it.t0[g], pol_q);
          tma_load_3d(qs + Q_HALF, &tmQ, &q_full[g][qb], 64, it.g * REP, it.rs + it.t0[g], pol_q);
          ++iq[g];
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      // Lane b < 4 reads the pool block of key block 4 j + b of the next K/V tile while lane 0
      // waits for a ring stage and issues the current tile's copies.
      const int last_pos = it.ctx0 + it.t0[0] + it.nt[0] - 1;  // tile 0 is the later one
      auto block_of = [&](int j) -> int {
        if (lane >= KT / 16) return 0;
        const int bi = j * (KT / 16) + lane;
        const int blk = bi < p.table_stride ? it.table[bi] : -1;
        if (blk < 0 || blk >= p.num_blocks) {
          // A block holding keys some row attends to must exist; past the last position
          // the keys are masked and any valid block serves as filler.
          if (bi * 16 <= last_pos) raise_status(p.status, B2_DEV_RANGE);
          return 0;
        }
        return blk;
      };
      int blk_next = block_of(0);
      for (int j = 0; j < it.n_kv[0] && ok; ++j, ++J) {
        const int blk_cur = blk_next;
        if (j + 1 < it.n_kv[0]) blk_next = block_of(j + 1);
        int y[KT / 16];
#pragma unroll
        for (int b = 0; b < KT / 16; ++b) y[b] = __shfl_sync(0xffffffffu, blk_cur, b) * 16;
        if (lane == 0) {
          const int st = J % ST;
          if (!mbar_wait(&kv_empty[st], ((uint32_t)(J / ST) & 1u) ^ 1u)) {
            raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
            ok = false;
          } else {
            uint8_t* sb = smem + (size_t)st * STAGE;
            mbar_arrive_expect_tx(&kv_full[st], STAGE);
#pragma unroll
            for (int b = 0; b < KT / 16; ++b) {
              tma_load_2d(sb + b * 2048, &tmK, &kv_full[st], it.g * HD, y[b], pol_kv);
              tma_load_2d(sb + HALF + b * 2048, &tmK, &kv_full[st], it.g * HD + 64, y[b], pol_kv);
              tma_load_2d(sb + 2 * HALF + b * 2048, &tmV, &kv_full[st], it.g * HD, y[b], pol_kv);
              tma_load_2d(sb + 3 * HALF + b * 2048, &tmV, &kv_full[st], it.g * HD + 64, y[b], pol_kv);
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
    }
    if (lane == 0) {
      // Copies still in flight (only after an aborted pipeline) land before the CTA exits.
      for (int g = 0; g < NG; ++g)
        for (int qb = 0; qb < 2; ++qb) {
          const int loads = (iq[g] + 1 - qb) / 2;  // copies made into buffer qb of group g
          if (loads > 0) mbar_wait(&q_full[g][qb], (uint32_t)(loads - 1) & 1u, 100000000ull);
        }
      for (int st = 0; st < ST && st < J; ++st) {
        const int last_i = st + ((J - 1 - st) / ST) * ST;
        mbar_wait(&kv_full[st], (uint32_t)(last_i / ST) & 1u, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer
    // The whole warp runs this control code, so that the operand descriptors stay in uniform
    // registers; one elected lane issues every tcgen05.mma and tcgen05.commit.  The tensor
    // cores queue only about one MMA ahead, so a wait on a barrier that has already completed
    // (a few hundred cycles for the answer) would leave them idle: the barrier of the next
    // step is tested before the current step's MMAs are issued (peek) and only waited for
    // when that answer was no.  S(n) into S buffer n & 1 needs no barrier of its own: the
    // softmax hands over P(n - 2) only after it has read S(n - 2), and PV(n - 2) is issued
    // (after that hand-over) before S(n).
    constexpr uint32_t idesc_s = instr_desc_bf16(ROWS, KT);
    constexpr uint32_t idesc_pv = instr_desc_bf16(ROWS, HD) | (1u << 16);  // B (V) MN-major
    int iq[NG] = {0, 0};  // Q tiles consumed per group
    int js[NG] = {0, 0};  // S tiles issued per group
    int jp[NG] = {0, 0};  // PV tiles issued per group
    int io[NG] = {0, 0};  // items started per group (O hand-offs)
    int qb[NG] = {0, 0};  // the Q buffer of the current item, per group
    int J = 0;
    bool ok = true;
    Peek pk_kv{0u, 0u, false}, pk_pf[NG] = {{0u, 0u, false}, {0u, 0u, false}};
    auto peek_pf = [&](int g) { peek(pk_pf[g], &p_full[g][jp[g] & 1], (uint32_t)(jp[g] >> 1) & 1u); };
    auto peek_kv = [&](int Jn) { peek(pk_kv, &kv_full[Jn % ST], (uint32_t)(Jn / ST) & 1u); };
    // O_g (+)= P_g V of the K/V tile in ring stage `st`; `first` starts the item's O; `ahead`
    // looks at the barrier of the step after this one, before this step's MMAs are issued.
    auto issue_pv = [&](int g, int st, bool first, auto&& ahead) -> bool {
      const int pb = jp[g] & 1;
      if (!__all_sync(0xffffffffu, wait_peeked(pk_pf[g], &p_full[g][pb], (uint32_t)(jp[g] >> 1) & 1u))) return false;
      if (first) {  // the previous item's O has been read out of TMEM
        if (!__all_sync(0xffffffffu, mbar_wait(&o_empty[g], ((uint32_t)io[g] & 1u) ^ 1u))) return false;
        ++io[g];
      }
      tc_fence_after();
      ahead();
      const uint32_t p_tmem = tmem + g * GROUP_COLS + COL_S + pb * KT;  // P(jp) in S buffer jp & 1
      const uint32_t v_addr = smem_u32(smem + (size_t)st * STAGE + 2 * HALF);
#pragma unroll
      for (int kk = 0; kk < KT / 16; ++kk)  // 16 keys per MMA: +8 TMEM columns of P, +2 KB of V rows
        if (elect_one())
          umma_bf16_ts(tmem + g * GROUP_COLS + COL_O, p_tmem + kk * 8,
                       smem_desc_sw128_mn(v_addr + kk * 2048, HALF, 1024), idesc_pv, (first && kk == 0) ? 0u : 1u);
      if (elect_one()) umma_commit(&pv_done[g][pb]);
      ++jp[g];
      return true;
    };
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
      const Item it = find_item<QT>(p, w, lane);
      if (!it.valid) continue;
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        if (it.nt[g] == 0 || !ok) continue;
        qb[g] = iq[g] & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&q_full[g][qb[g]], (uint32_t)(iq[g] >> 1) & 1u))) ok = false;
        ++iq[g];
      }
      for (int j = 0; j < it.n_kv[0] && ok; ++j, ++J) {
        const int st = J % ST;
        if (!__all_sync(0xffffffffu, wait_peeked(pk_kv, &kv_full[st], (uint32_t)(J / ST) & 1u))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + (size_t)st * STAGE);
        const int g_last = j < it.n_kv[1] ? 1 : 0;  // the last S batch of this tile
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          if (j >= it.n_kv[g]) continue;
          if (g == g_last) {  // next: PV_0 of tile j - 1, or the next K/V tile
            if (j >= 1) peek_pf(0);
            else peek_kv(J + 1);
          }
          const int b = js[g] & 1;
          const uint32_t q_addr = smem_u32(smem + OFF_Q + (g * 2 + qb[g]) * Q_BYTES);
#pragma unroll
          for (int half = 0; half < 2; ++half)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              if (elect_one())
                umma_bf16(tmem + g * GROUP_COLS + COL_S + b * KT, smem_desc_sw128(q_addr + half * Q_HALF) + 2 * kk,
                          smem_desc_sw128(k_addr + half * HALF) + 2 * kk, idesc_s, (half | kk) ? 1u : 0u);
          if (elect_one()) umma_commit(&s_full[g][b]);
          ++js[g];
          if (j == it.n_kv[g] - 1) {  // every S MMA of this item has read Q_g
            if (elect_one()) umma_commit(&q_empty[g][qb[g]]);
          }
        }
        if (j >= 1) {
          const int pst = (J - 1) % ST;
          const bool two = j - 1 < it.n_kv[1];  // group 1 also has a PV of tile j - 1
          if (ok) ok = issue_pv(0, pst, j == 1, [&] {
              if (two) peek_pf(1);
              else peek_kv(J + 1);
            });
          if (ok && two) ok = issue_pv(1, pst, j == 1, [&] { peek_kv(J + 1); });
          if (elect_one()) umma_commit(&kv_empty[pst]);  // both groups' S and PV of tile j - 1 are issued
        }
      }
      if (ok && it.n_kv[0] > 0) {  // the item's last tile (J is already the next tile's index)
        const int pst = (J - 1) % ST;
        const bool two = it.n_kv[1] == it.n_kv[0];
        const bool first = it.n_kv[0] == 1;
        ok = issue_pv(0, pst, first, [&] {
          if (two) peek_pf(1);
          else peek_kv(J);
        });
        if (ok && two) ok = issue_pv(1, pst, first, [&] { peek_kv(J); });
        if (elect_one()) umma_commit(&kv_empty[pst]);
      }
      if (!ok && lane == 0) raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
    }
    // every MMA issued by the elected lane has completed once drain_bar fires
    if (elect_one()) umma_commit(&drain_bar);
    mbar_wait(&drain_bar, 0, 100000000ull);
    __syncwarp();
  } else {
    // ---------------- softmax: one thread per MMA row of its group's Q tile
    const int sw = warp - 2;                 // 0..7
    const int grp = sw / kGroupWarps;        // 0: the later Q tile, 1: the one before
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int m = quarter * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16) + grp * GROUP_COLS;
    const int tk = m / REP, h = m % REP;
    int js = 0;  // S tiles consumed by this group (the PV of tile js - 1 is the latest issued)
    bool ok = true;
    Peek pk_s{0u, 0u, false};  // the next S tile, tested while this tile's P is written
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
      const Item it = find_item<QT>(p, w, lane);
      // this group's tile (selected without indexing, so the item stays in registers)
      const int nt = grp ? it.nt[1] : it.nt[0];
      const int t0 = grp ? it.t0[1] : it.t0[0];
      const int n_kv = grp ? it.n_kv[1] : it.n_kv[0];
      if (!it.valid || nt == 0) continue;
      const bool row_ok = tk < nt;
      const int pos = it.ctx0 + t0 + tk;  // this row's token position (the last key it attends to)
      float m_ref = -INFINITY, l_run = 0.f;
      for (int j = 0; j < n_kv; ++j, ++js) {
        const int b = js & 1;
        // warp-uniform verdicts: the TMEM loads and stores below are .sync.aligned
        if (!__all_sync(0xffffffffu, wait_peeked(pk_s, &s_full[grp][b], (uint32_t)(js >> 1) & 1u))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[64];
        tmem_ld32_nowait(trow + COL_S + b * KT, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        tmem_ld32_nowait(trow + COL_S + b * KT + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
        tmem_wait_ld();
        // raw scores; masked keys are -inf (scale_log2 > 0, so the maximum commutes with it)
        const int k0 = j * KT;
        float sv[64];
        if (row_ok && k0 + KT - 1 <= pos) {  // every key of the tile is visible (the common case)
#pragma unroll
          for (int e = 0; e < 64; ++e) sv[e] = __uint_as_float(sr[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 64; ++e) sv[e] = (row_ok && k0 + e <= pos) ? __uint_as_float(sr[e]) : -INFINITY;
        }
        float mx8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mx8[u] = sv[u];
#pragma unroll
        for (int e = 8; e < 64; e += 8)
#pragma unroll
          for (int u = 0; u < 8; ++u) mx8[u] = fmaxf(mx8[u], sv[e + u]);
#pragma unroll
        for (int u = 0; u < 4; ++u) mx8[u] = fmaxf(mx8[u], mx8[u + 4]);
        const float mx = fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])) * p.scale_log2;
        // the reference maximum: set by the first visible key, raised only by more than kRescale
        bool need = false;
        float corr = 1.f;
        if (m_ref == -INFINITY) {
          m_ref = mx;
        } else if (mx > m_ref + kRescale) {
          need = true;
          corr = exp2f(m_ref - mx);
        }
        if (__any_sync(0xffffffffu, need)) {
          // O must hold PV(js - 1) before it is rescaled (need implies j >= 1)
          if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[grp][(js - 1) & 1], (uint32_t)((js - 1) >> 1) & 1u))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            uint32_t o[32];
            tmem_ld32_nowait(trow + COL_O + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
            tmem_st32(trow + COL_O + c, o);
          }
          tmem_wait_st();
          if (need) {
            l_run *= corr;
            m_ref = mx;
          }
        }
        // P = exp2(s * scale_log2 - m_ref) in bf16 into the swizzled row of the group's P tile;
        // a row with nothing visible keeps p = 0 (m_ref = -inf is replaced by 0)
        const float m_sub = m_ref == -INFINITY ? 0.f : m_ref;
        float ls[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pw[32];  // the row's P in bf16 pairs: word w holds keys 2w (low half) and 2w + 1
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          // the next S tile this group consumes (in this item or the next): ask now, so that the
          // answer has arrived when this tile is done
          if (q == 2) peek(pk_s, &s_full[grp][(js + 1) & 1], (uint32_t)((js + 1) >> 1) & 1u);
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const int e = q * 8 + e2 * 2;
            const float p0 = ex2_approx(fmaf(sv[e], p.scale_log2, -m_sub));  // -inf gives 0
            const float p1 = ex2_approx(fmaf(sv[e + 1], p.scale_log2, -m_sub));
            ls[e2] += p0 + p1;
            __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
            pw[q * 4 + e2] = *reinterpret_cast<uint32_t*>(&h2);
          }
        }
        l_run += (ls[0] + ls[1]) + (ls[2] + ls[3]);
        // P over the first 32 columns of this S buffer (read above): the A operand of PV(js),
        // which the tensor cores run before S(js + 2) rewrites the buffer
        tmem_st32(trow + COL_S + b * KT, pw);
        tmem_wait_st();
        tc_fence_before();  // P and the rescaled O columns are read by the tensor cores
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[grp][b]);
      }
      if (!ok) break;
      // O / l to global memory once the item's last PV has completed; then O may be reused
      if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[grp][(js - 1) & 1], (uint32_t)((js - 1) >> 1) & 1u))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) +
                           (int64_t)(it.rs + t0 + tk) * p.ld_out + (int64_t)(it.g * REP + h) * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        uint32_t o[32];
        tmem_ld32_nowait(trow + COL_O + c, o);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int u = 0; u < 32; u += 8) {
            uint32_t wv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __nv_bfloat162 h2 = __floats2bfloat162_rn(__uint_as_float(o[u + 2 * e]) * inv,
                                                        __uint_as_float(o[u + 2 * e + 1]) * inv);
              wv[e] = *reinterpret_cast<uint32_t*>(&h2);
            }
            *reinterpret_cast<uint4*>(dst + c + u) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[grp]);
    }
    if (!ok && lane == 0) raise_status(p.status, B2_DEV_PIPE_TIMEOUT);
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
  const long items = (long)((n_rows / qt + n_seqs) / 2 + n_seqs) * nkv;  // an upper bound; the kernel counts exactly
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
