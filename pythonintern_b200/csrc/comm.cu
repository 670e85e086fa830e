// Tensor-parallel all-reduce over NVLink peer memory.
//
// Replaces the reference's gRPC all-reduce (engine/tensor_parallel/comm.py:72-154,
// buffer_codec.py:27-69, worker_node.py:107-125), in which every rank serialises
// its partial tensor, sends it to every peer and sums what arrives.  Here every
// rank owns one device allocation holding
//
//     [ data[0] | data[1] | flags[8][kMaxCtas] | ctrl{epoch, done} ]
//
// exported once through a CUDA IPC handle.  The row-parallel GEMM writes its
// partial straight into data[parity]; the reduction kernel then
//   1. raises flag[rank][cta] = epoch on every peer (st.release.sys),
//   2. waits, bounded by %globaltimer, for flag[peer][cta] == epoch from every
//      peer (ld.acquire.sys),
//   3. loads the partial of every rank directly over NVLink and sums in rank order
//      0..world-1 in float32 (so all ranks produce bit-identical results),
//   4. (fused variant) adds the float32 residual, writes it back, and applies the
//      next RMSNorm (layers.py:179-184).
// The epoch is a device-side counter advanced by the last CTA of every call, so
// CUDA-graph replays need no host bookkeeping.  Two data buffers alternate by call
// parity: a rank can only start overwriting data[p] after every peer has raised
// the flag of the following call, which it does only after finishing its reads of
// the previous use of data[p].
#include <cstring>
#include <new>

#include "common.cuh"
#include "gemm.cuh"

namespace b2 {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 128;

struct CommView {
  void* data[2][kMaxRanks];     // every rank's data (receive) buffers (own included)
  void* xn[2][kMaxRanks];       // every rank's all-gather buffers of normalised rows
  uint32_t* flags[kMaxRanks];   // every rank's flag array [2 phases][kMaxRanks][kMaxCtas]
  uint32_t* ctrl;               // own {epoch, done}
  int rank, world;
};

}  // namespace b2

struct b2_comm {
  int rank, world, device;
  size_t max_bytes, data_bytes;
  size_t off_data[2], off_xn[2], off_flags, off_ctrl, off_table, total;
  unsigned long long* scatter_table;  // device: [2 parities][kMaxRanks] peer data buffer addresses
  char* base;                       // own allocation
  char* peer_base[b2::kMaxRanks];   // mapped peers (own base at [rank])
  cudaIpcMemHandle_t handle;
  bool opened;
  bool local_peers;  // peers wired in-process by b2_comm_open_local (no IPC mappings to close)
};

namespace b2 {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Steps 1-2 of the protocol (flag set `phase`).  Returns false (and raises the status
// bit) on timeout.
__device__ bool comm_barrier(const CommView& v, uint32_t epoch, int64_t timeout_ns, int32_t* status,
                             int phase = 0) {
  __shared__ int s_ok;
  const int cta = blockIdx.x;
  const int pofs = phase * kMaxRanks * kMaxCtas;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < v.world) {
    __threadfence_system();
    st_release_sys(v.flags[threadIdx.x] + pofs + v.rank * kMaxCtas + cta, epoch);
  }
  if (threadIdx.x < v.world) {
    const uint32_t* f = v.flags[v.rank] + pofs + threadIdx.x * kMaxCtas + cta;
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
      if ((++it & 255) == 0 && (int64_t)(globaltimer_ns() - t0) > timeout_ns) {
        raise_status(status, B2_DEV_PEER_TIMEOUT);
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  return s_ok != 0;
}

// Last CTA to finish advances the epoch for the next call.
__device__ void comm_finish(const CommView& v) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(v.ctrl + 1, 1u);
    if (prev == gridDim.x - 1) {
      v.ctrl[1] = 0;
      v.ctrl[0] = v.ctrl[0] + 1;
      __threadfence();
    }
  }
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&o)[8]);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&o)[8]) {
  const uint4 raw = __ldcv(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = __uint_as_float(w[i] << 16);
    o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&o)[8]) {
  const float4 a = __ldcv(reinterpret_cast<const float4*>(p));
  const float4 b = __ldcv(reinterpret_cast<const float4*>(p) + 1);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
  o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}

template <typename T>
__device__ __forceinline__ void store8(T* dst, const float (&v)[8]);
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* dst, const float (&v)[8]) {
  uint4 o;
  uint32_t* w = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
    w[k] = *reinterpret_cast<uint32_t*>(&h2);
  }
  *reinterpret_cast<uint4*>(dst) = o;
}
template <>
__device__ __forceinline__ void store8<float>(float* dst, const float (&v)[8]) {
  reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// out[i] = sum_r data_r[parity][i], 8 elements per thread step.
template <typename T>
__global__ void allreduce_sum_kernel(CommView v, int parity, size_t n8, T* __restrict__ out,
                                     int64_t timeout_ns, int32_t* status) {
  const uint32_t epoch = v.ctrl[0] + 1;
  if (comm_barrier(v, epoch, timeout_ns, status)) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int r = 0; r < v.world; ++r) {
        float x[8];
        load8<T>(reinterpret_cast<const T*>(v.data[parity][r]) + i * 8, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += x[e];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) out[i * 8 + e] = from_f32<T>(acc[e]);
    }
  }
  comm_finish(v);
}

// h = residual + sum_r data_r[parity] (row-major [rows, dim]); y = rmsnorm(h) * w.
template <typename T>
__global__ void allreduce_rmsnorm_kernel(CommView v, int parity, int rows, int dim,
                                         const float* residual, float* h_out,
                                         const float* __restrict__ w, float eps, void* y,
                                         int y_dtype, int64_t timeout_ns, int32_t* status) {
  extern __shared__ float srow[];
  __shared__ float red[32];
  const uint32_t epoch = v.ctrl[0] + 1;
  if (comm_barrier(v, epoch, timeout_ns, status)) {
    const int nv = dim / 8;
    for (int row = blockIdx.x; row < rows; row += gridDim.x) {
      const size_t base = (size_t)row * dim;
      float ss = 0.f;
      for (int j = threadIdx.x; j < nv; j += blockDim.x) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int r = 0; r < v.world; ++r) {
          float x[8];
          load8<T>(reinterpret_cast<const T*>(v.data[parity][r]) + base + j * 8, x);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += x[e];
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float h = (residual ? residual[base + j * 8 + e] : 0.f) + acc[e];
          srow[j * 8 + e] = h;
          ss += h * h;
        }
      }
      ss = block_sum(ss, red);
      const float inv = rsqrtf(ss / (float)dim + eps);
      for (int c = threadIdx.x; c < dim; c += blockDim.x) {
        const float h = srow[c];
        if (h_out) h_out[base + c] = h;
        st_dyn(y, y_dtype, base + c, h * inv * w[c]);
      }
      __syncthreads();
    }
  }
  comm_finish(v);
}

// Second half of the row-parallel all-reduce with a row-sharded residual.  The partials
// were pushed by the row-parallel GEMM of every rank into this rank's data buffer as
// [src][R][dim] (R = rows per rank).  After barrier 0, each CTA takes owned rows
// (global row = rank * R + lr): h = h_slice + sum over src (rank order), h_slice = h,
// y = rmsnorm(h) * w, and pushes y into row `row` of EVERY rank's xn buffer.  Barrier 1
// then guarantees that all rows of the xn buffer are in place on every rank.
template <typename T>
__global__ void allreduce_rmsnorm_sharded_kernel(CommView v, int parity, int rows, int R, int dim,
                                                 float* h_slice, const float* __restrict__ w, float eps,
                                                 int64_t timeout_ns, int32_t* status) {
  __shared__ float red[32];
  const uint32_t epoch = v.ctrl[0] + 1;
  bool ok = comm_barrier(v, epoch, timeout_ns, status, 0);
  const int nv = dim / 8;
  if (ok) {
    const T* recv = reinterpret_cast<const T*>(v.data[parity][v.rank]);
    for (int lr = blockIdx.x; lr < R; lr += gridDim.x) {
      const int row = v.rank * R + lr;
      if (row >= rows) break;  // uniform across the CTA
      float hv[4][8];
      float ss = 0.f;
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int j = threadIdx.x + it * blockDim.x;
        if (j >= nv) continue;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int src = 0; src < v.world; ++src) {
          float x[8];
          load8<T>(recv + ((size_t)src * R + lr) * dim + j * 8, x);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += x[e];
        }
        float* hp = h_slice + (size_t)lr * dim + j * 8;
        const float4 h0 = *reinterpret_cast<const float4*>(hp);
        const float4 h1 = *reinterpret_cast<const float4*>(hp + 4);
        const float hr[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          hv[it][e] = hr[e] + acc[e];
          ss += hv[it][e] * hv[it][e];
        }
        *reinterpret_cast<float4*>(hp) = make_float4(hv[it][0], hv[it][1], hv[it][2], hv[it][3]);
        *reinterpret_cast<float4*>(hp + 4) = make_float4(hv[it][4], hv[it][5], hv[it][6], hv[it][7]);
      }
      ss = block_sum(ss, red);
      const float inv = rsqrtf(ss / (float)dim + eps);
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int j = threadIdx.x + it * blockDim.x;
        if (j >= nv) continue;
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = hv[it][e] * inv * w[j * 8 + e];
        for (int q = 0; q < v.world; ++q)  // all-gather by posted stores (own buffer included)
          store8<T>(reinterpret_cast<T*>(v.xn[parity][q]) + (size_t)row * dim + j * 8, o);
      }
      __syncthreads();
    }
  }
  if (ok) ok = comm_barrier(v, epoch, timeout_ns, status, 1);
  comm_finish(v);
}

static CommView make_view(const b2_comm* c) {
  CommView v{};
  v.rank = c->rank;
  v.world = c->world;
  for (int r = 0; r < c->world; ++r) {
    v.data[0][r] = c->peer_base[r] + c->off_data[0];
    v.data[1][r] = c->peer_base[r] + c->off_data[1];
    v.xn[0][r] = c->peer_base[r] + c->off_xn[0];
    v.xn[1][r] = c->peer_base[r] + c->off_xn[1];
    v.flags[r] = reinterpret_cast<uint32_t*>(c->peer_base[r] + c->off_flags);
  }
  v.ctrl = reinterpret_cast<uint32_t*>(c->base + c->off_ctrl);
  return v;
}

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Fills the device table of every rank's data-buffer address (as seen from this rank).
static int fill_scatter_table(b2_comm* c) {
  unsigned long long t[2 * kMaxRanks] = {0};
  for (int par = 0; par < 2; ++par)
    for (int r = 0; r < c->world; ++r)
      t[par * kMaxRanks + r] = (unsigned long long)(uintptr_t)(c->peer_base[r] + c->off_data[par]);
  int dev = 0;
  B2_TRY_CUDA(cudaGetDevice(&dev));
  B2_TRY_CUDA(cudaSetDevice(c->device));
  cudaError_t e = cudaMemcpy(c->scatter_table, t, sizeof(t), cudaMemcpyHostToDevice);
  cudaSetDevice(dev);
  if (e != cudaSuccess) return fail(B2_ECUDA, "scatter table upload: %s", cudaGetErrorString(e));
  return B2_OK;
}

}  // namespace b2

extern "C" {

size_t b2_comm_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int b2_comm_create(int rank, int world_size, size_t max_bytes, b2_comm** out) {
  B2_CHECK_ARG(out, "b2_comm_create: null out");
  B2_CHECK_ARG(world_size >= 1 && world_size <= b2::kMaxRanks, "b2_comm_create: world_size %d not in [1, 8]", world_size);
  B2_CHECK_ARG(rank >= 0 && rank < world_size, "b2_comm_create: rank %d out of range", rank);
  B2_CHECK_ARG(max_bytes > 0, "b2_comm_create: max_bytes must be > 0");
  b2_comm* c = new (std::nothrow) b2_comm();
  if (!c) return b2::fail(B2_EINVAL, "b2_comm_create: out of host memory");
  c->rank = rank;
  c->world = world_size;
  B2_TRY_CUDA(cudaGetDevice(&c->device));
  c->max_bytes = max_bytes;
  c->data_bytes = b2::align_up(max_bytes, 4096);
  c->off_data[0] = 0;
  c->off_data[1] = c->data_bytes;
  c->off_xn[0] = 2 * c->data_bytes;
  c->off_xn[1] = 3 * c->data_bytes;
  c->off_flags = 4 * c->data_bytes;
  c->off_ctrl = c->off_flags + b2::align_up((size_t)2 * b2::kMaxRanks * b2::kMaxCtas * sizeof(uint32_t), 256);
  c->off_table = c->off_ctrl + 256;
  c->total = c->off_table + 256;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&c->base), c->total);
  if (e != cudaSuccess) {
    delete c;
    return b2::fail(B2_ECUDA, "b2_comm_create: cudaMalloc(%zu): %s", (size_t)0, cudaGetErrorString(e));
  }
  e = cudaMemset(c->base + c->off_flags, 0, c->total - c->off_flags);
  if (e == cudaSuccess) e = cudaMemset(c->base, 0, 4 * c->data_bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&c->handle, c->base);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(c->base);
    delete c;
    return b2::fail(B2_ECUDA, "b2_comm_create: %s", cudaGetErrorString(e));
  }
  for (int r = 0; r < b2::kMaxRanks; ++r) c->peer_base[r] = nullptr;
  c->peer_base[rank] = c->base;
  c->scatter_table = reinterpret_cast<unsigned long long*>(c->base + c->off_table);
  c->opened = world_size == 1;
  c->local_peers = false;
  if (world_size == 1) {
    const int rc = b2::fill_scatter_table(c);
    if (rc) {
      cudaFree(c->base);
      delete c;
      return rc;
    }
  }
  *out = c;
  return B2_OK;
}

int b2_comm_export_handle(b2_comm* comm, void* handle, size_t len) {
  B2_CHECK_ARG(comm && handle && len >= sizeof(cudaIpcMemHandle_t), "b2_comm_export_handle: bad arguments");
  memcpy(handle, &comm->handle, sizeof(cudaIpcMemHandle_t));
  return B2_OK;
}

int b2_comm_open_peers(b2_comm* comm, const void* all_handles, size_t len) {
  B2_CHECK_ARG(comm && all_handles, "b2_comm_open_peers: null argument");
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  B2_CHECK_ARG(len >= hb * comm->world, "b2_comm_open_peers: %zu bytes given, %zu needed", len, hb * comm->world);
  B2_CHECK_ARG(!comm->opened || comm->world == 1, "b2_comm_open_peers: already opened");
  const char* h = static_cast<const char*>(all_handles);
  for (int r = 0; r < comm->world; ++r) {
    if (r == comm->rank) continue;
    cudaIpcMemHandle_t ph;
    memcpy(&ph, h + r * hb, hb);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, ph, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != comm->rank && comm->peer_base[q]) {
          cudaIpcCloseMemHandle(comm->peer_base[q]);
          comm->peer_base[q] = nullptr;
        }
      return b2::fail(B2_ECUDA, "b2_comm_open_peers: rank %d handle: %s", r, cudaGetErrorString(e));
    }
    comm->peer_base[r] = static_cast<char*>(p);
  }
  comm->opened = true;
  return b2::fill_scatter_table(comm);
}

int b2_comm_open_local(b2_comm* const* comms, int n) {
  B2_CHECK_ARG(comms && n >= 1 && n <= b2::kMaxRanks, "b2_comm_open_local: bad arguments");
  for (int i = 0; i < n; ++i) {
    B2_CHECK_ARG(comms[i] && comms[i]->world == n && comms[i]->rank == i,
                 "b2_comm_open_local: comms[%d] must be rank %d of a world of %d", i, i, n);
    for (int j = 0; j < i; ++j)
      B2_CHECK_ARG(comms[i]->device != comms[j]->device,
                   "b2_comm_open_local: ranks %d and %d share device %d (one GPU per rank)", j, i, comms[i]->device);
  }
  int dev = 0;
  B2_TRY_CUDA(cudaGetDevice(&dev));
  for (int i = 0; i < n; ++i) {
    B2_TRY_CUDA(cudaSetDevice(comms[i]->device));
    for (int j = 0; j < n; ++j) {
      if (j == i) continue;
      int can = 0;
      B2_TRY_CUDA(cudaDeviceCanAccessPeer(&can, comms[i]->device, comms[j]->device));
      if (!can) {
        cudaSetDevice(dev);
        return b2::fail(B2_ENOTSUP, "b2_comm_open_local: device %d cannot access device %d", comms[i]->device, comms[j]->device);
      }
      cudaError_t e = cudaDeviceEnablePeerAccess(comms[j]->device, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
      } else if (e != cudaSuccess) {
        cudaSetDevice(dev);
        return b2::fail(B2_ECUDA, "b2_comm_open_local: enable peer access %d->%d: %s", comms[i]->device, comms[j]->device, cudaGetErrorString(e));
      }
    }
  }
  B2_TRY_CUDA(cudaSetDevice(dev));
  for (int i = 0; i < n; ++i) {
    for (int j = 0; j < n; ++j) comms[i]->peer_base[j] = comms[j]->base;
    comms[i]->opened = true;
    comms[i]->local_peers = true;
    const int rc = b2::fill_scatter_table(comms[i]);
    if (rc) return rc;
  }
  return B2_OK;
}

int b2_comm_buffer(b2_comm* comm, int parity, void** ptr) {
  B2_CHECK_ARG(comm && ptr && (parity == 0 || parity == 1), "b2_comm_buffer: bad arguments");
  *ptr = comm->base + comm->off_data[parity];
  return B2_OK;
}

int b2_comm_xn_buffer(b2_comm* comm, int parity, void** ptr) {
  B2_CHECK_ARG(comm && ptr && (parity == 0 || parity == 1), "b2_comm_xn_buffer: bad arguments");
  *ptr = comm->base + comm->off_xn[parity];
  return B2_OK;
}

int b2_comm_destroy(b2_comm* comm) {
  if (!comm) return B2_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaSetDevice(comm->device);
  cudaDeviceSynchronize();
  if (!comm->local_peers)
    for (int r = 0; r < comm->world; ++r)
      if (r != comm->rank && comm->peer_base[r]) cudaIpcCloseMemHandle(comm->peer_base[r]);
  cudaFree(comm->base);
  cudaSetDevice(dev);
  delete comm;
  return B2_OK;
}

int b2_allreduce_sum(b2_comm* comm, int parity, size_t count, int dtype, void* out,
                     int64_t timeout_ns, int32_t* status, b2_stream_t stream) {
  B2_CHECK_ARG(comm && comm->opened, "b2_allreduce_sum: communicator not opened");
  B2_CHECK_ARG(parity == 0 || parity == 1, "b2_allreduce_sum: parity must be 0 or 1");
  B2_CHECK_ARG(b2::valid_dtype(dtype), "b2_allreduce_sum: bad dtype");
  B2_CHECK_ARG(count % 8 == 0, "b2_allreduce_sum: count must be a multiple of 8");
  B2_CHECK_ARG(count * b2::dtype_bytes(dtype) <= comm->max_bytes, "b2_allreduce_sum: %zu elements exceed the buffer", count);
  B2_CHECK_ARG(out && ((uintptr_t)out % 16) == 0, "b2_allreduce_sum: out must be 16-byte aligned");
  if (count == 0) return B2_OK;
  const b2::CommView v = b2::make_view(comm);
  const size_t n8 = count / 8;
  int grid = (int)((n8 + 255) / 256);
  if (grid > b2::kMaxCtas) grid = b2::kMaxCtas;
  if (grid < 1) grid = 1;
  if (dtype == B2_BF16)
    b2::allreduce_sum_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(v, parity, n8, (__nv_bfloat16*)out, timeout_ns, status);
  else
    b2::allreduce_sum_kernel<float><<<grid, 256, 0, stream>>>(v, parity, n8, (float*)out, timeout_ns, status);
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

int b2_allreduce_rmsnorm(b2_comm* comm, int parity, int rows, int dim, int dtype,
                         const float* residual, float* h_out, const float* norm_w, float eps,
                         void* y, int y_dtype, int64_t timeout_ns, int32_t* status,
                         b2_stream_t stream) {
  B2_CHECK_ARG(comm && comm->opened, "b2_allreduce_rmsnorm: communicator not opened");
  B2_CHECK_ARG(parity == 0 || parity == 1, "b2_allreduce_rmsnorm: parity must be 0 or 1");
  B2_CHECK_ARG(b2::valid_dtype(dtype) && b2::valid_dtype(y_dtype), "b2_allreduce_rmsnorm: bad dtype");
  B2_CHECK_ARG(rows >= 0 && dim > 0 && dim % 8 == 0 && dim <= 12288, "b2_allreduce_rmsnorm: bad dim %d", dim);
  B2_CHECK_ARG((size_t)rows * dim * b2::dtype_bytes(dtype) <= comm->max_bytes, "b2_allreduce_rmsnorm: payload exceeds the buffer");
  if (rows == 0) return B2_OK;
  B2_CHECK_ARG(norm_w && y, "b2_allreduce_rmsnorm: null pointer");
  const b2::CommView v = b2::make_view(comm);
  const int grid = rows < b2::kMaxCtas ? rows : b2::kMaxCtas;
  const int threads = dim >= 4096 ? 512 : 256;
  const size_t smem = (size_t)dim * sizeof(float);
  if (dtype == B2_BF16) {
    if (smem > 48 * 1024)
      B2_TRY_CUDA(cudaFuncSetAttribute(b2::allreduce_rmsnorm_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    b2::allreduce_rmsnorm_kernel<__nv_bfloat16><<<grid, threads, smem, stream>>>(
        v, parity, rows, dim, residual, h_out, norm_w, eps, y, y_dtype, timeout_ns, status);
  } else {
    if (smem > 48 * 1024)
      B2_TRY_CUDA(cudaFuncSetAttribute(b2::allreduce_rmsnorm_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    b2::allreduce_rmsnorm_kernel<float><<<grid, threads, smem, stream>>>(
        v, parity, rows, dim, residual, h_out, norm_w, eps, y, y_dtype, timeout_ns, status);
  }
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

int b2_row_parallel_linear(b2_comm* comm, int parity, const void* x, int64_t ldx, int M, int K, const void* w,
                           int N, int dtype, void* workspace, size_t workspace_bytes, int32_t* status,
                           b2_stream_t stream) {
  B2_CHECK_ARG(comm && comm->opened, "b2_row_parallel_linear: communicator not opened");
  B2_CHECK_ARG(parity == 0 || parity == 1, "b2_row_parallel_linear: parity must be 0 or 1");
  B2_CHECK_ARG(b2::valid_dtype(dtype), "b2_row_parallel_linear: bad dtype");
  B2_CHECK_ARG(M >= 0 && K > 0 && N > 0 && ldx >= K, "b2_row_parallel_linear: bad sizes");
  if (M == 0) return B2_OK;
  B2_CHECK_ARG(x && w, "b2_row_parallel_linear: null pointer");
  const int R = (M + comm->world - 1) / comm->world;
  B2_CHECK_ARG((size_t)comm->world * R * N * b2::dtype_bytes(dtype) <= comm->max_bytes,
               "b2_row_parallel_linear: %d x %d partial exceeds the communicator buffer", M, N);
  b2::Scatter sc{comm->scatter_table + parity * b2::kMaxRanks, R, comm->rank, comm->world};
  if (dtype == B2_F32) return b2::gemm_simt(x, ldx, M, K, w, nullptr, N, nullptr, nullptr, N, dtype, dtype, stream, &sc);
  b2::GemmSeg seg{w, N, 0};
  return b2::gemm_tc(x, ldx, M, K, &seg, 1, b2::kEpiStore, nullptr, nullptr, N, dtype, workspace, workspace_bytes,
                     status, stream, &sc);
}

int b2_allreduce_rmsnorm_sharded(b2_comm* comm, int parity, int rows, int dim, int dtype, float* h_slice,
                                 const float* norm_w, float eps, int64_t timeout_ns, int32_t* status,
                                 b2_stream_t stream) {
  B2_CHECK_ARG(comm && comm->opened, "b2_allreduce_rmsnorm_sharded: communicator not opened");
  B2_CHECK_ARG(parity == 0 || parity == 1, "b2_allreduce_rmsnorm_sharded: parity must be 0 or 1");
  B2_CHECK_ARG(b2::valid_dtype(dtype), "b2_allreduce_rmsnorm_sharded: bad dtype");
  B2_CHECK_ARG(rows >= 0 && dim > 0 && dim % 8 == 0 && dim <= 8 * 4 * 512,
               "b2_allreduce_rmsnorm_sharded: bad dim %d", dim);
  if (rows == 0) return B2_OK;
  const int R = (rows + comm->world - 1) / comm->world;
  B2_CHECK_ARG((size_t)comm->world * R * dim * b2::dtype_bytes(dtype) <= comm->max_bytes,
               "b2_allreduce_rmsnorm_sharded: payload exceeds the buffer");
  B2_CHECK_ARG(norm_w && (h_slice || comm->rank * R >= rows), "b2_allreduce_rmsnorm_sharded: null pointer");
  B2_CHECK_ARG(((uintptr_t)h_slice % 16) == 0 && ((uintptr_t)norm_w % 16) == 0,
               "b2_allreduce_rmsnorm_sharded: h_slice and norm_w must be 16-byte aligned");
  const b2::CommView v = b2::make_view(comm);
  const int grid = R < b2::kMaxCtas ? R : b2::kMaxCtas;
  int threads = 64;
  while (threads < 512 && threads * 4 < dim / 8) threads *= 2;
  if (dtype == B2_BF16)
    b2::allreduce_rmsnorm_sharded_kernel<__nv_bfloat16><<<grid, threads, 0, stream>>>(
        v, parity, rows, R, dim, h_slice, norm_w, eps, timeout_ns, status);
  else
    b2::allreduce_rmsnorm_sharded_kernel<float><<<grid, threads, 0, stream>>>(
        v, parity, rows, R, dim, h_slice, norm_w, eps, timeout_ns, status);
  B2_TRY_CUDA(cudaGetLastError());
  return B2_OK;
}

}  // extern "C"
