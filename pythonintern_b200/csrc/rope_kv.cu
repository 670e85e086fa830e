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
__device__ __forceinline__ void ld4(const T* p, float (&v)[4]) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  } else {
    const uint2 a = *reinterpret_cast<const uint2*>(p);
    v[0] = __uint_as_float(a.x << 16); v[1] = __uint_as_float(a.x & 0xffff0000u);
    v[2] = __uint_as_float(a.y << 16); v[3] = __uint_as_float(a.y & 0xffff0000u);
  }
}
template <typename T>
__device__ __forceinline__ void st4(T* p, const float (&v)[4]) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&a);
    o.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = o;
  }
}

// grid = (work blocks, tokens).  Work item i of a token: i < (nq + nkv) * hd/8 rotates
// pairs d..d+3 (with partners d+hd/2..) of one q or k head; the next nkv * hd/8 items
// copy 8 value elements each.
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
  pdl_wait();
  pdl_trigger();
  const int tok = blockIdx.y;
  const int half = hd >> 1;
  const int64_t p = rope_pos[tok];
  const int64_t ps = store_pos ? store_pos[tok] : p;
  const int row = table_index ? table_index[tok] : tok;
  const bool pos_ok = p >= 0 && p < max_seq_len;
  int64_t blk = -1;
  if (ps >= 0 && (ps / bs) < table_stride) blk = tables[(int64_t)row * table_stride + ps / bs];
  const bool slot_ok = blk >= 0 && blk < num_blocks;
  if (blockIdx.x == 0 && threadIdx.x == 0 && !(pos_ok && slot_ok)) raise_status(status, B2_DEV_RANGE);
  if (!pos_ok) return;
  const int64_t slot_off = slot_ok ? layer_elems * layer + ((blk * bs + ps % bs) * nkv) * (int64_t)hd : 0;
  const T* src = qkv + (int64_t)tok * ld_qkv;
  const int per_head = hd / 8;
  const int n_rot = (nq + nkv) * per_head;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n_rot) {
    const int h = i / per_head, d = (i % per_head) * 4;
    const T* xh = src + (int64_t)h * hd;
    float x1[4], x2[4], c1[4], s1[4], c2[4], s2[4], o1[4], o2[4];
    ld4<T>(xh + d, x1);
    ld4<T>(xh + d + half, x2);
    ld4<float>(cos_t + p * hd + d, c1);
    ld4<float>(sin_t + p * hd + d, s1);
    ld4<float>(cos_t + p * hd + d + half, c2);
    ld4<float>(sin_t + p * hd + d + half, s2);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      // out[d] = x1*cos[d] + (-x2)*sin[d];  out[d+half] = x2*cos[d+half] + x1*sin[d+half]
      o1[e] = __fadd_rn(__fmul_rn(x1[e], c1[e]), __fmul_rn(-x2[e], s1[e]));
      o2[e] = __fadd_rn(__fmul_rn(x2[e], c2[e]), __fmul_rn(x1[e], s2[e]));
    }
    T* dst;
    if (h < nq) {
      dst = q_out + ((int64_t)tok * nq + h) * hd;
    } else {
      if (!slot_ok) return;
      dst = k_cache + slot_off + (int64_t)(h - nq) * hd;
    }
    st4<T>(dst + d, o1);
    st4<T>(dst + d + half, o2);
  } else if (i < n_rot + nkv * per_head) {
    if (!slot_ok) return;
    const int j = (i - n_rot) * 8;  // values are stored unrotated
    const T* vsrc = src + (int64_t)(nq + nkv) * hd + j;
    T* vdst = v_cache + slot_off + j;
    float a[4], b[4];
    ld4<T>(vsrc, a);
    ld4<T>(vsrc + 4, b);
    st4<T>(vdst, a);
    st4<T>(vdst + 4, b);
  }
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
  B2_CHECK_ARG(head_dim % 8 == 0, "b2_rope_kv_write: head_dim must be a multiple of 8");
  const size_t esz = b2::dtype_bytes(dtype);
  B2_CHECK_ARG(((uintptr_t)qkv % 16) == 0 && ((ld_qkv * esz) % 16) == 0 && ((uintptr_t)q_out % 16) == 0 &&
                   ((uintptr_t)k_cache % 16) == 0 && ((uintptr_t)v_cache % 16) == 0 && ((uintptr_t)cos % 16) == 0 &&
                   ((uintptr_t)sin % 16) == 0,
               "b2_rope_kv_write: buffers must be 16-byte aligned");
  B2_CHECK_ARG(n_tokens <= 65535, "b2_rope_kv_write: n_tokens %d > 65535", n_tokens);
  const int64_t layer_elems = (int64_t)num_blocks * block_size * nkv * head_dim;
  const int threads = 128;
  const int work = (nq + 2 * nkv) * (head_dim / 8);
  const dim3 grid((work + threads - 1) / threads, n_tokens);
  if (dtype == B2_BF16) {
    using T = __nv_bfloat16;
    B2_TRY_CUDA(b2::launch_pdl((b2::rope_kv_write_kernel<T>), grid, dim3(threads), 0, stream,
        (const T*)qkv, ld_qkv, nq, nkv, head_dim, rope_pos, store_pos, table_index, block_tables,
        table_stride, num_blocks, block_size, cos, sin, max_seq_len, (T*)q_out, (T*)k_cache,
        (T*)v_cache, layer_elems, layer, status));
  } else {
    B2_TRY_CUDA(b2::launch_pdl((b2::rope_kv_write_kernel<float>), grid, dim3(threads), 0, stream,
        (const float*)qkv, ld_qkv, nq, nkv, head_dim, rope_pos, store_pos, table_index,
        block_tables, table_stride, num_blocks, block_size, cos, sin, max_seq_len, (float*)q_out,
        (float*)k_cache, (float*)v_cache, layer_elems, layer, status));
  }
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}
