// Internal declarations shared by the GEMM translation units.
#pragma once
#include "common.cuh"

namespace b2 {

// silu(x) = x / (1 + exp(-x)), float32 (torch.nn.functional.silu, engine/model/mlp.py:82)
__device__ __forceinline__ float silu_f32(float x) { return x / (1.f + expf(-x)); }

// Epilogue kinds of the tensor-core GEMM.
enum GemmEpi { kEpiStore = 0, kEpiSwiglu = 1 };

// One output segment of a grouped launch: rows [0, n) of the packed [n, K] weight w,
// written to output columns [col_off, col_off + n).
struct GemmSeg {
  const void* w;
  int n;
  int col_off;
};

// Reduce-scatter destination of a row-parallel GEMM: output row m goes to rank
// o = m / rows_per_rank, at row (src * rows_per_rank + m % rows_per_rank) of the receive
// slot whose device address is table[(*epoch % 3) * 8 + o] (peer memory for o != src).
// world == 0: plain output.
struct Scatter {
  const unsigned long long* table;
  const unsigned int* epoch;
  int rows_per_rank, src, world;
};

int gemm_simt(const void* x, int64_t ldx, int M, int K, const void* w0, const void* w1, int N,
              const float* bias, void* y, int64_t ldy, int dtype, int y_dtype, cudaStream_t s,
              const Scatter* sc = nullptr);

// Address of output element (m, col) for a plain or scattered destination.
__device__ __forceinline__ void* out_base(void* y, int y_dtype, int64_t ldy, const unsigned long long* table,
                                          const unsigned int* epoch, int R, int src, int world, int64_t m,
                                          int64_t col, int64_t* idx) {
  if (world > 0) {
    const int o = (int)(m / R);
    *idx = ((int64_t)src * R + (m - (int64_t)o * R)) * ldy + col;
    return reinterpret_cast<void*>(table[(*epoch % 3u) * 8u + o]);
  }
  *idx = m * ldy + col;
  return y;
}

// Deferred RMSNorm options of the tcgen05 GEMM (world size 1; see b2_linear_residual_norm).
struct RowNorm {
  const float* row_ss;  // consumer: per-row tile sums of h^2 [M, n_ss]
  int n_ss;
  float ss_scale, ss_eps;  // 1 / hidden size, epsilon
  float* res_h;            // producer: float32 residual [M, ldh] (updated in place)
  int64_t ldh;
  const float* norm_w;     // producer: RMSNorm weight [N]
  void* z;                 // producer: bf16 h * norm_w [M, ldz]
  int64_t ldz;
  float* ss_out;           // producer: tile sums of h^2 [M, N / 128]
};

// Fused RoPE + paged KV write epilogue of the q|k|v GEMM (head_dim 128: one 128-row weight
// tile per head; see b2_linear_qkv_rope_kv).  Mirrors rope_kv_write_kernel argument for argument.
struct RopeKV {
  int nq, nkv;
  const int64_t* rope_pos;
  const int64_t* store_pos;
  const int32_t* table_index;
  const int32_t* tables;
  int table_stride, num_blocks, block_size, max_seq_len;
  const float* cos_t;
  const float* sin_t;
  void* q_out;
  void* k_cache;
  void* v_cache;
  int64_t layer_off;  // elements from the pool start to this layer
};

// bf16 tcgen05 GEMM. For kEpiStore: nseg segments (1..3) concatenated along N.
// For kEpiSwiglu: segs[0] = gate, segs[1] = up, both with n = N.
size_t gemm_tc_workspace_bytes(int M, int n_total, int K, int epi);
// rn: deferred RMSNorm (consumer and/or producer); the producer needs the split-K cluster
// plan, a single segment, N % 128 == 0 and no SwiGLU, else B2_ENOTSUP before any launch.
int gemm_tc(const void* x, int64_t ldx, int M, int K, const GemmSeg* segs, int nseg, int epi,
            const float* bias, void* y, int64_t ldy, int y_dtype, void* ws, size_t ws_bytes,
            int32_t* status, cudaStream_t s, const Scatter* sc = nullptr, const RowNorm* rn = nullptr,
            const RopeKV* rk = nullptr);
// Returns true when the tensor-core kernel supports the shape (K % 8 == 0, 16-byte aligned rows).
bool gemm_tc_supported(const void* x, int64_t ldx, int K, const GemmSeg* segs, int nseg);

}  // namespace b2
