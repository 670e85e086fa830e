// Rotary embedding of q/k and the paged KV-cache write.
//
// Restates engine/model/attention.py:46-63 (rotate-half RoPE) and :166-184 with
// engine/model/kv_cache.py:35-43, :85-100 (slot = table[p / bs], p % bs).
// The rotation uses the float32 cos/sin tables built on the host with the
// reference's formula, and explicit round-to-nearest multiplies and adds (no FMA
// contraction), so the float32 path reproduces the reference's two-rounding
// ``x*cos + rotate_half(x)*sin`` bit for bit.
#include "common.cuh"

namespace b2 {

template <typename T>
__global__ void rope_kv_write_kernel(const T* __restrict__ qkv, int64_t ld_qkv, int nq, int nkv,
                                     int hd, const int64_t* __restrict__ rope_pos,
                                     const int64_t* __restrict__ store_pos,
                                     const int32_t* __restrict__ table_index,
                                     const int32_t* __restrict__ tables, int table_stride,
                                     int num_blocks, int bs, const float* __restrict__ cos_t,
                                     const float* __restrict__ sin_t, int max_seq_len,
                                     T* __restrict__ q_out, T* __restrict__ k_cache,
                                     T* __restrict__ v_cache, int64_t layer_elems, int layer,
                                     int32_t* status) {
  const int tok = blockIdx.x;
  const int half = hd >> 1;
  const int64_t p = rope_pos[tok];
  const int64_t ps = store_pos ? store_pos[tok] : p;
  const int row = table_index ? table_index[tok] : tok;
  const bool pos_ok = p >= 0 && p < max_seq_len;
  int64_t blk = -1;
  if (ps >= 0 && (ps / bs) < table_stride) blk = tables[(int64_t)row * table_stride + ps / bs];
  const bool slot_ok = blk >= 0 && blk < num_blocks;
  if (threadIdx.x == 0 && !(pos_ok && slot_ok)) raise_status(status, B2_DEV_RANGE);
  if (!pos_ok) return;

  const T* src = qkv + (int64_t)tok * ld_qkv;
  const float* c = cos_t + p * hd;
  const float* s = sin_t + p * hd;
  const int64_t slot_off = slot_ok ? layer_elems * layer + ((blk * bs + ps % bs) * nkv) * (int64_t)hd : 0;

  // Rotated heads: q heads then k heads, one (head, pair) per thread iteration.
  const int rot_pairs = (nq + nkv) * half;
  for (int i = threadIdx.x; i < rot_pairs; i += blockDim.x) {
    const int h = i / half, d = i % half;
    const T* xh = src + h * hd;
    const float x1 = to_f32(xh[d]);
    const float x2 = to_f32(xh[d + half]);
    // out[d]      = x1*cos[d]      + (-x2)*sin[d]
    // out[d+half] = x2*cos[d+half] + ( x1)*sin[d+half]
    const float o1 = __fadd_rn(__fmul_rn(x1, c[d]), __fmul_rn(-x2, s[d]));
    const float o2 = __fadd_rn(__fmul_rn(x2, c[d + half]), __fmul_rn(x1, s[d + half]));
    if (h < nq) {
      T* dst = q_out + ((int64_t)tok * nq + h) * hd;
      dst[d] = from_f32<T>(o1);
      dst[d + half] = from_f32<T>(o2);
    } else if (slot_ok) {
      T* dst = k_cache + slot_off + (int64_t)(h - nq) * hd;
      dst[d] = from_f32<T>(o1);
      dst[d + half] = from_f32<T>(o2);
    }
  }
  if (!slot_ok) return;
  // Values are stored unrotated.
  const T* vsrc = src + (int64_t)(nq + nkv) * hd;
  T* vdst = v_cache + slot_off;
  for (int i = threadIdx.x; i < nkv * hd; i += blockDim.x) vdst[i] = vsrc[i];
}

}  // namespace b2

extern "C" int b2_rope_kv_write(const void* qkv, int64_t ld_qkv, int n_tokens, int nq, int nkv,
                                int head_dim, const int64_t* rope_pos, const int64_t* store_pos,
                                const int32_t* table_index, const int32_t* block_tables,
                                int table_stride, int num_blocks, int block_size, const float* cos,
                                const float* sin, int max_seq_len, void* q_out, void* k_cache,
                                void* v_cache, int layer, int dtype, int32_t* status,
                                b2_stream_t stream) {
  B2_CHECK_ARG(n_tokens >= 0 && nq > 0 && nkv > 0 && head_dim > 0 && (head_dim % 2) == 0,
               "b2_rope_kv_write: bad head sizes");
  B2_CHECK_ARG(ld_qkv >= (int64_t)(nq + 2 * nkv) * head_dim, "b2_rope_kv_write: ld_qkv too small");
  B2_CHECK_ARG(num_blocks > 0 && block_size > 0 && table_stride > 0 && layer >= 0 && max_seq_len > 0,
               "b2_rope_kv_write: bad cache geometry");
  B2_CHECK_ARG(b2::valid_dtype(dtype), "b2_rope_kv_write: bad dtype");
  if (n_tokens == 0) return B2_OK;
  B2_CHECK_ARG(qkv && rope_pos && block_tables && cos && sin && q_out && k_cache && v_cache,
               "b2_rope_kv_write: null pointer");
  const int64_t layer_elems = (int64_t)num_blocks * block_size * nkv * head_dim;
  const int threads = 128;
  if (dtype == B2_BF16) {
    using T = __nv_bfloat16;
    b2::rope_kv_write_kernel<T><<<n_tokens, threads, 0, stream>>>(
        (const T*)qkv, ld_qkv, nq, nkv, head_dim, rope_pos, store_pos, table_index, block_tables,
        table_stride, num_blocks, block_size, cos, sin, max_seq_len, (T*)q_out, (T*)k_cache,
        (T*)v_cache, layer_elems, layer, status);
  } else {
    b2::rope_kv_write_kernel<float><<<n_tokens, threads, 0, stream>>>(
        (const float*)qkv, ld_qkv, nq, nkv, head_dim, rope_pos, store_pos, table_index,
        block_tables, table_stride, num_blocks, block_size, cos, sin, max_seq_len, (float*)q_out,
        (float*)k_cache, (float*)v_cache, layer_elems, layer, status);
  }
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}
