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

#include "common.cuh"

namespace b2 {

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

template <typename T, int HD, int REP>
__global__ void __launch_bounds__(kAttnWarps * 32) paged_attn_simt_kernel(AttnParams p) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int LPT = HD / VEC;  // lanes per token row
  constexpr int G = 32 / LPT;    // token rows per warp step
  constexpr int CH = 4;          // tokens per lane group per chunk
  static_assert(LPT >= 1 && LPT <= 32 && (32 % LPT) == 0, "head_dim/vector mismatch");

  __shared__ float sm_m[kAttnWarps][REP], sm_l[kAttnWarps][REP];
  __shared__ float sm_acc[kAttnWarps][REP][HD];
  __shared__ int sm_flag;
  __shared__ float red[32];

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
    for (int w = 1; w < kAttnWarps; ++w) all = fmaxf(all, red[w]);
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
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_m[w][r]);
      float L = 0.f, A = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
          const float f = safe_exp2_diff(sm_m[w][r], M);
          L += sm_l[w][r] * f;
          A += sm_acc[w][r][d] * f;
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
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_m[w][r]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float f = safe_exp2_diff(sm_m[w][r], M);
        L += sm_l[w][r] * f;
        A += sm_acc[w][r][d] * f;
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
  switch (rep) {
    case 1: paged_attn_simt_kernel<T, HD, 1><<<grid, kAttnWarps * 32, 0, s>>>(p); break;
    case 2: paged_attn_simt_kernel<T, HD, 2><<<grid, kAttnWarps * 32, 0, s>>>(p); break;
    case 4: paged_attn_simt_kernel<T, HD, 4><<<grid, kAttnWarps * 32, 0, s>>>(p); break;
    case 8: paged_attn_simt_kernel<T, HD, 8><<<grid, kAttnWarps * 32, 0, s>>>(p); break;
    default: return fail(B2_ENOTSUP, "b2_paged_attention: nq/nkv = %d not supported (1, 2, 4, 8)", rep);
  }
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
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
  B2_CHECK_ARG(n_rows >= 0 && nq > 0 && nkv > 0 && nq % nkv == 0, "b2_paged_attention: bad head counts");
  B2_CHECK_ARG(b2::valid_dtype(dtype), "b2_paged_attention: bad dtype");
  B2_CHECK_ARG(num_blocks > 0 && block_size > 0 && table_stride > 0 && layer >= 0,
               "b2_paged_attention: bad cache geometry");
  B2_CHECK_ARG(num_splits >= 1 && num_splits <= 1024, "b2_paged_attention: num_splits %d out of [1, 1024]", num_splits);
  B2_CHECK_ARG(ld_q >= (int64_t)nq * head_dim && ld_out >= (int64_t)nq * head_dim,
               "b2_paged_attention: row strides too small");
  if (n_rows == 0) return B2_OK;
  B2_CHECK_ARG(q && k_cache && v_cache && block_tables && ctx_lens && out, "b2_paged_attention: null pointer");
  B2_CHECK_ARG(n_rows <= 65535, "b2_paged_attention: n_rows %d > 65535", n_rows);
  const size_t esz = b2::dtype_bytes(dtype);
  B2_CHECK_ARG(((uintptr_t)q % 16) == 0 && ((ld_q * esz) % 16) == 0 && ((uintptr_t)k_cache % 16) == 0 &&
                   ((uintptr_t)v_cache % 16) == 0,
               "b2_paged_attention: q/cache must be 16-byte aligned");
  b2::AttnWs lay = b2::attn_ws_layout(n_rows, nq, nkv, head_dim, num_splits);
  b2::AttnParams p{};
  if (num_splits > 1) {
    B2_CHECK_ARG((size_t)n_rows * nkv <= b2::kAttnCounterSlots,
                 "b2_paged_attention: n_rows * nkv = %d exceeds %zu with num_splits > 1", n_rows * nkv,
                 b2::kAttnCounterSlots);
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
  if (dtype == B2_BF16) return b2::launch_hd<__nv_bfloat16>(head_dim, rep, p, grid, stream);
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
  void* scratch = nullptr;
  if (num_splits > 1) {
    B2_CHECK_ARG(n_rows >= 0 && nq > 0 && nkv > 0 && head_dim > 0 && num_splits <= 1024,
                 "b2_paged_attention_noalloc: bad sizes");
    const size_t need = b2_paged_attention_workspace_bytes(n_rows, nq, nkv, head_dim, num_splits);
    B2_CHECK_ARG(need <= b2::kNoAllocScratchBytes,
                 "b2_paged_attention_noalloc: this call needs %zu bytes of split scratch but the static "
                 "array holds %zu; use fewer splits or rows, or b2_paged_attention with a workspace",
                 need, b2::kNoAllocScratchBytes);
    const int rc = b2::noalloc_scratch(&scratch);
    if (rc) return rc;
    // The array keeps the previous call's contents: zero the split counters this call uses.
    if (n_rows > 0) B2_TRY_CUDA(cudaMemsetAsync(scratch, 0, (size_t)n_rows * nkv * sizeof(int), stream));
  }
  return b2_paged_attention(q, ld_q, n_rows, nq, nkv, head_dim, k_cache, v_cache, layer, num_blocks, block_size,
                            block_tables, table_stride, table_index, ctx_lens, compat_pad, scale, out, ld_out,
                            dtype, scratch, scratch ? b2::kNoAllocScratchBytes : 0, num_splits, status, stream);
}

}  // extern "C"
