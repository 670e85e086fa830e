/*
 * b2tp.h - C ABI of libb2tp.so, the B200 (sm_100a) kernels behind the
 * tensor-parallel decoder-layer forward of the pythonintern inference engine.
 *
 * Conventions
 *  - Every entry point returns an int status (B2_OK on success).  A failing
 *    call leaves a message retrievable with b2_last_error() (per host thread).
 *  - All device work is enqueued asynchronously on the caller's stream; no entry
 *    point synchronises or allocates device memory, except the communicator's
 *    create/destroy calls, which set up and tear down its symmetric buffers.
 *  - All pointers are device pointers unless stated.  Tensors are row-major and
 *    caller owned.  Element types are given by B2_F32 / B2_BF16 codes.
 *  - Linear weights are passed PACKED as [N, K] with K contiguous, i.e. the
 *    transpose of the reference's [in, out] parameter layout
 *    (engine/tensor_parallel/layers.py:55-61, :123-129).  The Python layer keeps
 *    the reference's [in, out] parameter as a transposed view of that buffer.
 *  - `status` (nullable) is a caller-owned device int32 that kernels OR error
 *    bits into (B2_DEV_*); it is never cleared by the library.
 *
 * Citations name the reference file:line each entry point replaces, relative to
 * the reference project root.
 */
#ifndef B2TP_H
#define B2TP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* b2_stream_t; /* identical to cudaStream_t */

enum b2_status_code {
  B2_OK = 0,
  B2_EINVAL = 1,   /* bad argument (shape, dtype, alignment, null pointer) */
  B2_ETIMEOUT = 2, /* a peer did not arrive within the timeout (comm.py:99-107) */
  B2_ECUDA = 3,    /* CUDA runtime error */
  B2_ENOTSUP = 4,  /* shape/dtype combination not implemented */
  B2_ERANGE = 5    /* index out of range (position, block table entry, token id) */
};

enum b2_dtype { B2_F32 = 0, B2_BF16 = 1 };

/* Device-side error bits ORed into *status by kernels. */
enum b2_device_error {
  B2_DEV_RANGE = 1,        /* position >= max_seq_len, block index past the table, bad block id, bad token id */
  B2_DEV_PIPE_TIMEOUT = 2, /* an in-kernel pipeline wait (mbarrier) ran out of its bound */
  B2_DEV_PEER_TIMEOUT = 4  /* a peer flag was not raised before the all-reduce timeout */
};

/* ---------------------------------------------------------------- library */
int b2_abi_version(void);
const char* b2_status_name(int status);
/* Copies the calling thread's last error message into buf (always NUL terminated). */
int b2_last_error(char* buf, size_t len);

/* ---------------------------------------------------------------- embedding
 * out[i, :] = table[ids[i], :]                       (engine/model/llama.py:150)
 * ids out of [0, vocab) write zeros and raise B2_DEV_RANGE. */
int b2_embedding(const int64_t* ids, int n, const void* table, int vocab, int dim, int dtype,
                 void* out, int out_dtype, int32_t* status, b2_stream_t stream);

/* ---------------------------------------------------------------- RMSNorm
 * h = x (+ residual);  if h_out: h_out = h;  y = h * rsqrt(mean(h^2) + eps) * weight
 * (engine/tensor_parallel/layers.py:179-184 and the residual adds of
 *  engine/model/llama.py:61,70,73,75,164).  residual/h_out may be NULL; x, residual
 * and h_out may alias.  weight is float32 [dim].  With y == NULL (and h_out set) the
 * call is the bare residual add h_out = x + residual (llama.py:75). */
int b2_rmsnorm(const void* x, int x_dtype, const void* residual, int residual_dtype, void* h_out,
               int h_dtype, const float* weight, float eps, void* y, int y_dtype, int rows, int dim,
               b2_stream_t stream);

/* ---------------------------------------------------------------- linear
 * y[m, n] = sum_k x[m, k] * w[n, k] (+ bias[n])
 * ColumnParallelLinear.forward (engine/tensor_parallel/layers.py:78-86) and the
 * partial GEMM of RowParallelLinear.forward (layers.py:147-152).
 * dtype: type of x and w (B2_BF16 runs on tcgen05 tensor cores, B2_F32 runs the
 * float32 FFMA kernel); y_dtype: B2_F32 or dtype.  workspace: scratch of
 * b2_linear_workspace_bytes() bytes (may be 0 for some shapes), zero-filled
 * once by the caller before its first use; the kernels leave it ready for reuse.
 * Calls that share a workspace must be stream ordered. */
size_t b2_linear_workspace_bytes(int M, int N, int K, int dtype);
int b2_linear(const void* x, int64_t ldx, int M, int K, const void* w, int N, const float* bias,
              void* y, int64_t ldy, int dtype, int y_dtype, void* workspace, size_t workspace_bytes,
              int32_t* status, b2_stream_t stream);

/* Fused q/k/v projections of DistributedAttention (engine/model/attention.py:156-158):
 * y[:, 0:Nq] = x.Wq^T, y[:, Nq:Nq+Nk] = x.Wk^T, y[:, Nq+Nk:Nq+Nk+Nv] = x.Wv^T (ldy >= Nq+Nk+Nv). */
int b2_linear_qkv(const void* x, int64_t ldx, int M, int K, const void* wq, int Nq, const void* wk,
                  int Nk, const void* wv, int Nv, void* y, int64_t ldy, int dtype, void* workspace,
                  size_t workspace_bytes, int32_t* status, b2_stream_t stream);

/* Fused gate/up projections + SwiGLU of DistributedMLP (engine/model/mlp.py:80-82):
 * y[m, j] = silu(x[m].w_gate[j]) * (x[m].w_up[j]),  j < N. */
int b2_linear_swiglu(const void* x, int64_t ldx, int M, int K, const void* w_gate, const void* w_up,
                     int N, void* y, int64_t ldy, int dtype, void* workspace,
                     size_t workspace_bytes, int32_t* status, b2_stream_t stream);

/* Deferred RMSNorm at world size 1 (bf16, M <= 512 rows).  Together these replace
 * RowParallelLinear.forward + the residual add + the next RMSNorm (layers.py:147-162,
 * 179-184; llama.py:70-75) followed by the next ColumnParallelLinear / SwiGLU
 * (attention.py:156-158, mlp.py:80-82), without a separate normalisation kernel:
 *   b2_linear_residual_norm: h [M, N] float32 (row stride ldh) += x @ w^T, then
 *     z [M, N] bf16 = h * norm_w (not yet divided by the RMS) and ss [M, N/128] = the
 *     sum of h^2 over each 128-column tile.  N % 128 == 0.  Returns B2_ENOTSUP, before
 *     launching anything, when the shape gets no split-K cluster plan (the caller then
 *     uses b2_linear + b2_rmsnorm).  Workspace: b2_linear_workspace_bytes(M, N, K).
 *   b2_linear_qkv_rownorm / b2_linear_swiglu_rownorm: b2_linear_qkv / b2_linear_swiglu on
 *     x = z whose output row m is scaled by rsqrt(sum_j ss[m * n_ss + j] / dim + eps),
 *     i.e. the GEMM of the normalised rows (the two SwiGLU halves both scaled). */
int b2_linear_residual_norm(const void* x, int64_t ldx, int M, int K, const void* w, int N, float* h, int64_t ldh,
                            const float* norm_w, void* z, int64_t ldz, float* ss, void* workspace,
                            size_t workspace_bytes, int32_t* status, b2_stream_t stream);
int b2_linear_qkv_rownorm(const void* x, int64_t ldx, int M, int K, const void* wq, int Nq, const void* wk, int Nk,
                          const void* wv, int Nv, void* y, int64_t ldy, const float* ss, int n_ss, int dim, float eps,
                          void* workspace, size_t workspace_bytes, int32_t* status, b2_stream_t stream);
int b2_linear_swiglu_rownorm(const void* x, int64_t ldx, int M, int K, const void* w_gate, const void* w_up, int N,
                             void* y, int64_t ldy, const float* ss, int n_ss, int dim, float eps, void* workspace,
                             size_t workspace_bytes, int32_t* status, b2_stream_t stream);

/* q|k|v GEMM with RoPE and the paged KV write in its epilogue: b2_linear_qkv (or, with ss
 * set, b2_linear_qkv_rownorm) followed by b2_rope_kv_write, without the intermediate
 * [M, (nq + 2 nkv) * 128] buffer (attention.py:156-158 then :46-63, :166-184).  The
 * outputs are bit-identical to the two calls.  head_dim must be 128 and M <= 512; returns
 * B2_ENOTSUP, before launching anything, otherwise or when the shape gets no split-K
 * cluster plan (the caller then makes the two calls).  bf16 only. */
int b2_linear_qkv_rope_kv(const void* x, int64_t ldx, int M, int K, const void* wq, const void* wk, const void* wv,
                          int nq, int nkv, int head_dim, const float* ss, int n_ss, int dim, float eps,
                          const int64_t* rope_pos, const int64_t* store_pos, const int32_t* table_index,
                          const int32_t* block_tables, int table_stride, int num_blocks, int block_size,
                          const float* cos, const float* sin, int max_seq_len, void* q_out, void* k_cache,
                          void* v_cache, int layer, void* workspace, size_t workspace_bytes, int32_t* status,
                          b2_stream_t stream);

/* ---------------------------------------------------------------- RoPE + paged KV write
 * For token i (0 <= i < n_tokens) with row = table_index ? table_index[i] : i:
 *   q_out[i, h, :]   = rope(qkv[i, q-head h], rope_pos[i])                 (attention.py:46-63,161)
 *   k_cache[layer, blk, off, g, :] = rope(qkv[i, k-head g], rope_pos[i])   (attention.py:162,166-184)
 *   v_cache[layer, blk, off, g, :] = qkv[i, v-head g]                      (kv_cache.py:85-100)
 * where (blk, off) = (block_tables[row*table_stride + p/block_size], p % block_size),
 * p = store_pos ? store_pos[i] : rope_pos[i]                               (kv_cache.py:35-43).
 * qkv rows hold [q heads | k heads | v heads] (nq+2*nkv)*head_dim wide with row stride ld_qkv.
 * cos/sin: float32 [max_seq_len, head_dim] tables.  Caches: [L, num_blocks, block_size, nkv, head_dim].
 * Out-of-range positions or table entries skip the token and raise B2_DEV_RANGE. */
int b2_rope_kv_write(const void* qkv, int64_t ld_qkv, int n_tokens, int nq, int nkv, int head_dim,
                     const int64_t* rope_pos, const int64_t* store_pos, const int32_t* table_index,
                     const int32_t* block_tables, int table_stride, int num_blocks, int block_size,
                     const float* cos, const float* sin, int max_seq_len, void* q_out,
                     void* k_cache, void* v_cache, int layer, int dtype, int32_t* status,
                     b2_stream_t stream);

/* ---------------------------------------------------------------- paged attention
 * One query token per row b (0 <= b < n_rows), attending to the first ctx_lens[b]
 * tokens of the paged cache through block-table row table_index ? table_index[b] : b.
 * q: [n_rows, nq, head_dim] (row stride ld_q); out: [n_rows, nq*head_dim] (row stride ld_out).
 * GQA: q head h reads kv head h / (nq/nkv)                     (attention.py:66-76,208-209)
 * out = softmax(q.K^T * scale) V                               (attention.py:216-228)
 * compat_pad != 0 reproduces the reference's decode batch: every row is zero-padded
 * to the longest ctx_lens in the call WITHOUT a mask (attention.py:190-203), so
 * (max_ctx - ctx) zero scores join each softmax denominator.  compat_pad == 0 gives
 * the masked result (used for causal prompt attention, attention.py:219-222).
 * num_splits (>= 1) is the number of CTAs that share one (row, kv head): each takes an
 * equal run of KV blocks and the last one to finish merges the partial softmax states.
 * workspace: b2_paged_attention_workspace_bytes(n_rows, nq, nkv, head_dim, num_splits)
 * bytes (0 when num_splits == 1), zero-filled once before first use. */
size_t b2_paged_attention_workspace_bytes(int n_rows, int nq, int nkv, int head_dim, int num_splits);
int b2_paged_attention(const void* q, int64_t ld_q, int n_rows, int nq, int nkv, int head_dim,
                       const void* k_cache, const void* v_cache, int layer, int num_blocks,
                       int block_size, const int32_t* block_tables, int table_stride,
                       const int32_t* table_index, const int32_t* ctx_lens, int compat_pad,
                       float scale, void* out, int64_t ld_out, int dtype, void* workspace,
                       size_t workspace_bytes, int num_splits, int32_t* status, b2_stream_t stream);

/* Allocation-free variant of b2_paged_attention (no counterpart in the reference).
 * For callers that cannot allocate device memory: a host that reaches this library
 * only through the plain C ABI (cgo, JNI, ctypes) and has no device allocator of its
 * own, or a worker whose device memory was handed in full to another runtime's pool
 * at start-up, where a cudaMalloc would fail or fragment that pool.  The split
 * scratch lives in a 4 MiB static array inside the library (every GPU that loads the
 * library holds it until the process exits); calls needing more are rejected with
 * B2_EINVAL.  The first call on a device looks up the array's device address with
 * cudaGetSymbolAddress; make that first call before any stream capture.  All calls
 * share the array, so calls that overlap on the GPU (different streams without
 * ordering) race; order them on one stream.  Allocates nothing: no cudaMalloc or
 * cudaFree.  Arguments and result are those of b2_paged_attention. */
int b2_paged_attention_noalloc(const void* q, int64_t ld_q, int n_rows, int nq, int nkv, int head_dim,
                               const void* k_cache, const void* v_cache, int layer, int num_blocks,
                               int block_size, const int32_t* block_tables, int table_stride,
                               const int32_t* table_index, const int32_t* ctx_lens, int compat_pad,
                               float scale, void* out, int64_t ld_out, int dtype, int num_splits,
                               int32_t* status, b2_stream_t stream);

/* Causal prefill attention for any number of sequences in one call.
 * Replaces the prefill branch of DistributedAttention.forward (engine/model/attention.py:
 * 166-174 store, :211-228 scores with the causal mask of :219-222), which the reference
 * runs one sequence per forward (engine/worker/execution_engine.py:85-111).
 * Rows [seq_start[s], seq_start[s+1]) of q (and out) are the tokens of sequence s, at
 * positions seq_ctx0[s] + (row - seq_start[s]) (seq_ctx0 null: 0); row r attends to the
 * keys at positions 0..pos(r) of its sequence, read from the pool through block-table
 * row s (their K/V must already be stored, e.g. by b2_rope_kv_write).  seq_start must be
 * non-decreasing with seq_start[0] >= 0 and seq_start[n_seqs] <= n_rows.
 * bf16 only, block_size 16, head_dim 32/64/128, nq/nkv in {1,2,4,8}; other shapes return
 * B2_ENOTSUP (the per-row b2_paged_attention covers them).  Block ids outside the pool
 * or sequences outside [0, n_rows) set B2_DEV_RANGE in *status and are skipped. */
int b2_prefill_attention(const void* q, int64_t ld_q, int n_rows, int nq, int nkv, int head_dim,
                         const void* k_cache, const void* v_cache, int layer, int num_blocks, int block_size,
                         const int32_t* block_tables, int table_stride, const int32_t* seq_start,
                         const int32_t* seq_ctx0, int n_seqs, float scale, void* out, int64_t ld_out, int dtype,
                         int32_t* status, b2_stream_t stream);

/* The same causal prefill attention on the 5th-generation tensor cores: S = Q K^T and
 * P V accumulated in TMEM by tcgen05.mma, Q/K/V tiles fed by TMA from q and the paged pool,
 * softmax and the output rescaling on the CUDA cores.  Replaces the same reference code as
 * b2_prefill_attention (engine/model/attention.py:166-174, :211-228).  bf16, head_dim 128,
 * block_size 16, nq/nkv in {1,2,4,8}; q/out rows and the pool 16-byte aligned; other shapes
 * return B2_EINVAL or B2_ENOTSUP without launching.  b2_prefill_attention uses this kernel
 * for the shapes it serves. */
int b2_prefill_attention_tc(const void* q, int64_t ld_q, int n_rows, int nq, int nkv, int head_dim,
                            const void* k_cache, const void* v_cache, int layer, int num_blocks, int block_size,
                            const int32_t* block_tables, int table_stride, const int32_t* seq_start,
                            const int32_t* seq_ctx0, int n_seqs, float scale, void* out, int64_t ld_out, int dtype,
                            int32_t* status, b2_stream_t stream);

/* ---------------------------------------------------------------- greedy sampling
 * out[r] = first index of the maximum of logits[r, 0:cols]   (execution_engine.py:103,133) */
int b2_argmax(const float* logits, int64_t ld, int rows, int cols, int64_t* out, b2_stream_t stream);

/* ---------------------------------------------------------------- communicator
 * Replaces DistributedCommunicator (engine/tensor_parallel/comm.py:27-166), its
 * wire codec (engine/tensor_parallel/buffer_codec.py:27-69) and the receive side
 * (engine/worker/worker_node.py:107-125) with NVLink peer memory: each rank owns
 * two symmetric data buffers and a flag array, exported through CUDA IPC handles
 * that the host exchanges once (over any control plane), then reads its peers'
 * buffers directly inside the reduction kernel.
 * Protocol: every all-reduce call carries the next epoch of a device-side counter;
 * each CTA raises its flag on every peer and waits, with a bound of timeout_ns
 * (globaltimer), for the matching flag of every peer.  A timed-out wait raises
 * B2_DEV_PEER_TIMEOUT in *status and the communicator must then be destroyed. */
typedef struct b2_comm b2_comm;
size_t b2_comm_handle_bytes(void);
int b2_comm_create(int rank, int world_size, size_t max_bytes, b2_comm** out);
int b2_comm_export_handle(b2_comm* comm, void* handle, size_t len);
/* all_handles: world_size handles of b2_comm_handle_bytes() each, in rank order. */
int b2_comm_open_peers(b2_comm* comm, const void* all_handles, size_t len);
/* In-process alternative to IPC (the reference's register_in_memory_peer,
 * comm.py:51-53): comms[i] is rank i of a world of n, each created with its own
 * device current; peers are wired with direct peer pointers.  All ranks must be on
 * distinct GPUs. */
int b2_comm_open_local(b2_comm* const* comms, int n);
/* Device pointer of this rank's symmetric data buffer `parity` (0 or 1). */
int b2_comm_buffer(b2_comm* comm, int parity, void** ptr);
int b2_comm_destroy(b2_comm* comm);

/* out[i] = sum over ranks r = 0..world-1 (in that order) of buffer_r[parity][i]
 * (comm.py:72-118, all_reduce_sum).  out must not be a symmetric buffer: peers may
 * still be reading them while this rank writes its result. */
int b2_allreduce_sum(b2_comm* comm, int parity, size_t count, int dtype, void* out,
                     int64_t timeout_ns, int32_t* status, b2_stream_t stream);

/* Fused row-parallel epilogue: h = residual + sum_r buffer_r[parity][rows, dim]
 * (ranks in order), then y = rmsnorm(h) * norm_w.  residual/h_out are float32 and
 * may alias.  (RowParallelLinear all-reduce layers.py:155-158 + llama.py:70,73,75 +
 * RMSNorm layers.py:179-184 of the next norm.) */
int b2_allreduce_rmsnorm(b2_comm* comm, int parity, int rows, int dim, int dtype,
                         const float* residual, float* h_out, const float* norm_w, float eps,
                         void* y, int y_dtype, int64_t timeout_ns, int32_t* status,
                         b2_stream_t stream);

/* Row-parallel linear fused with the reduce-scatter of its all-reduce
 * (RowParallelLinear.forward, engine/tensor_parallel/layers.py:147-158): the partial
 * y = x.w^T is computed on this rank and row m of it is stored, straight from the GEMM
 * epilogue, into the current receive slot of rank m / R (R = ceil(M / world)) at row
 * (this rank * R + m % R); rows owned by peers travel over NVLink while the GEMM runs.
 * The next b2_allreduce_rmsnorm_sharded call on the same communicator completes it. */
int b2_row_parallel_linear(b2_comm* comm, const void* x, int64_t ldx, int M, int K, const void* w, int N,
                           int dtype, void* workspace, size_t workspace_bytes, int32_t* status,
                           b2_stream_t stream);

/* Completes the all-reduce of b2_row_parallel_linear for a row-sharded residual
 * (comm.py:72-118 + llama.py:70,75 + the next RMSNorm, layers.py:179-184): this rank
 * owns rows [rank*R, rank*R + R) of the [rows, dim] activations and keeps their float32
 * residual in h_slice [R, dim].  h_slice += the sum over ranks (rank order) of their
 * partial rows; the rows are normalised by norm_w and pushed to every rank, and on
 * return y [rows, dim] holds all normalised rows on every rank.  No flags: every
 * element's arrival is detected in sentinel-filled rotating slots, each wait bounded
 * by timeout_ns. */
int b2_allreduce_rmsnorm_sharded(b2_comm* comm, int rows, int dim, int dtype, float* h_slice, const float* norm_w,
                                 float eps, void* y, int64_t timeout_ns, int32_t* status, b2_stream_t stream);

/* Greedy token per row over a vocab-parallel lm_head: replaces torch.argmax over the
 * replicated logits (execution_engine.py:103,133 on the lm_head of llama.py:168-170).
 * logits [rows, cols] float32 (row stride ld) are this rank's logits for vocabulary ids
 * [vocab_offset, vocab_offset + cols); the ranks exchange (max, index) per row through
 * the communicator and every rank writes the global argmax (first index of the maximum,
 * NaN wins, as torch.argmax) to out [rows] int64.  rows <= 4096.  Each wait is bounded
 * by timeout_ns (device bit B2_DEV_PEER_TIMEOUT on expiry). */
int b2_argmax_allgather(b2_comm* comm, const float* logits, int64_t ld, int rows, int cols, int64_t vocab_offset,
                        int64_t* out, int64_t timeout_ns, int32_t* status, b2_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* B2TP_H */
