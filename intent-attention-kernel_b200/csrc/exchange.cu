// Peer-memory exchange of partial blocks for multi-GPU split-KV decode, and
// the CUDA IPC helpers that map the ranks' exchange areas into each process.
//
// Area of one rank (device memory of its GPU), for world W and block size
// BF = rows * (head_dim + 2) floats padded to BS (a multiple of 64 floats):
//   float  blocks[2][W][BS]      receive arrays, one per parity
//   float  staging[BS]           this rank's partial block (written by the decode)
//   uint32 flags[2][W]           arrival epoch of each sender, per parity
//   uint32 push_count[2]         CTAs of this rank's push kernel that finished
//   uint32 epoch                 last epoch this rank pushed (device-side, so a
//                                captured CUDA graph can replay the steps)
// A push reads epoch e, copies the staging block into slot `rank` of every
// rank's blocks[(e+1) & 1] with plain stores over NVLink, and its last CTA
// (after a system-scope fence) raises flag[(e+1) & 1][rank] = e+1 in every
// area and advances epoch.  The merge waits, bounded in time, for all W flags
// of that parity in its own area and then LSE-merges the W blocks.
#include <algorithm>
#include <cstring>

#include "iak_internal.cuh"

namespace iak {
namespace {

constexpr int kPushThreads = 256;

__host__ __device__ inline int64_t block_stride(int64_t rows, int D) { return exchange_block_stride(rows, D); }
__host__ __device__ inline size_t staging_offset(int world, int64_t rows, int D) {
  return exchange_staging_offset(world, rows, D);
}
__host__ __device__ inline size_t flags_offset(int world, int64_t rows, int D) {
  return exchange_flags_offset(world, rows, D);
}

struct PushParams {
  float* areas[IAK_MAX_PEERS];
  int rank, world;
  int64_t bs;          // block stride (floats)
  int64_t n4;          // float4 per block copy
  size_t staging_off;  // byte offsets inside an area
  size_t flags_off;
};

__device__ __forceinline__ uint32_t* area_flags(float* area, size_t off) {
  return reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(area) + off);
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(kPushThreads) push_kernel(const PushParams p) {
  float* own = p.areas[p.rank];
  uint32_t* own_flags = area_flags(own, p.flags_off);
  // epoch word: read by every CTA before the last one advances it
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(own_flags + 2 * p.world + 2) + 1u;
  const int parity = static_cast<int>(epoch & 1u);
  const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const char*>(own) + p.staging_off);
  for (int r = 0; r < p.world; ++r) {
    float4* dst = reinterpret_cast<float4*>(p.areas[r] + (static_cast<int64_t>(parity) * p.world + p.rank) * p.bs);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < p.n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
      dst[i] = src[i];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* count = own_flags + 2 * p.world + parity;
    if (atomicAdd(count, 1u) == gridDim.x - 1) {
      // every CTA's stores are fenced: publish the block to every rank, then advance the epoch
      *count = 0u;
      __threadfence_system();
      for (int r = 0; r < p.world; ++r)
        st_release_sys(area_flags(p.areas[r], p.flags_off) + parity * p.world + p.rank, epoch);
      own_flags[2 * p.world + 2] = epoch;
    }
  }
}

// Bounded wait (timeout_ns of wall time) by thread 0 for every sender's flag of the
// current epoch (the one this rank just published), then the LSE merge of the W
// blocks of that parity into out, one CTA per row.  A CTA whose wait runs out sets
// *status and merges whatever arrived.
__global__ void exchange_merge_kernel(const float* area, const uint32_t* flags, int world, int64_t rows, int D,
                                      int64_t bs, void* out, int out_dtype, int64_t out_row_stride,
                                      uint32_t* status, uint64_t timeout_ns) {
  extern __shared__ float w_s[];
  __shared__ float stat[2];
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(flags + 2 * world + 2);
  const uint32_t* f = flags + (epoch & 1u) * world;
  if (threadIdx.x == 0) {
    const uint64_t t0 = global_ns();
    bool late = false;
    for (int r = 0; r < world && !late; ++r) {
      unsigned ns = 32;
      while (ld_acquire_sys(f + r) != epoch) {
        if (global_ns() - t0 > timeout_ns) {
          late = true;
          if (status) atomicExch(status, 1u);
          break;
        }
        __nanosleep(ns);
        if (ns < 512) ns <<= 1;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < world) (void)ld_acquire_sys(f + threadIdx.x);   // acquire for every reading warp
  __syncthreads();
  const float* blocks = area + static_cast<int64_t>(epoch & 1u) * world * bs;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    if (threadIdx.x < 32) {
      float M = -INFINITY;
      for (int s = threadIdx.x; s < world; s += 32) {
        const float* b = blocks + s * bs;
        if (b[rows + r] > 0.f) M = fmaxf(M, b[r]);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      float L = 0.f;
      for (int s = threadIdx.x; s < world; s += 32) {
        const float* b = blocks + s * bs;
        const float ls = b[rows + r];
        const float w = (ls > 0.f && M != -INFINITY) ? expf(b[r] - M) : 0.f;
        w_s[s] = w;
        L += ls * w;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
      if (threadIdx.x == 0) {
        stat[0] = M;
        stat[1] = L;
      }
    }
    __syncthreads();
    const float L = stat[1];
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float A = 0.f;
      for (int s = 0; s < world; ++s) {
        const float w = w_s[s];
        if (w != 0.f) A = fmaf(blocks[s * bs + 2 * rows + r * D + d], w, A);
      }
      store_from_float(out, out_dtype, r * out_row_stride + d, L > 0.f ? A / L : 0.f);
    }
    __syncthreads();
  }
}

int check_exchange(const iak_peer_exchange* x) {
  if (!x) return fail(IAK_ERR_INVALID_ARG, "null exchange descriptor");
  if (x->world < 1 || x->world > IAK_MAX_PEERS) return fail(IAK_ERR_INVALID_ARG, "world %d outside 1..%d", x->world, IAK_MAX_PEERS);
  if (x->rank < 0 || x->rank >= x->world) return fail(IAK_ERR_INVALID_ARG, "rank %d outside world %d", x->rank, x->world);
  if (x->rows < 0 || x->head_dim <= 0) return fail(IAK_ERR_INVALID_ARG, "bad block shape");
  for (int r = 0; r < x->world; ++r)
    if (!x->areas[r] || reinterpret_cast<uintptr_t>(x->areas[r]) % 256)
      return fail(IAK_ERR_INVALID_ARG, "exchange area of rank %d is NULL or not 256-byte aligned", r);
  return IAK_OK;
}

}  // namespace
}  // namespace iak

using namespace iak;

extern "C" {

int iak_exchange_area_bytes(int32_t world, int64_t rows, int32_t head_dim, size_t* bytes) {
  if (!bytes) return fail(IAK_ERR_INVALID_ARG, "bytes is NULL");
  if (world < 1 || world > IAK_MAX_PEERS || rows < 0 || head_dim <= 0) return fail(IAK_ERR_INVALID_ARG, "bad exchange shape");
  *bytes = flags_offset(world, rows, head_dim) + 256;
  return IAK_OK;
}

float* iak_exchange_staging_ptr(void* area, int32_t world, int64_t rows, int32_t head_dim) {
  if (!area || world < 1 || world > IAK_MAX_PEERS || rows < 0 || head_dim <= 0) return nullptr;
  return reinterpret_cast<float*>(static_cast<char*>(area) + staging_offset(world, rows, head_dim));
}

int iak_exchange_push(const iak_peer_exchange* x, void* stream) {
  int st = check_exchange(x);
  if (st) return st;
  PushParams p;
  std::memset(&p, 0, sizeof(p));
  for (int r = 0; r < x->world; ++r) p.areas[r] = static_cast<float*>(x->areas[r]);
  p.rank = x->rank; p.world = x->world;
  p.bs = block_stride(x->rows, x->head_dim);
  p.n4 = (x->rows * (static_cast<int64_t>(x->head_dim) + 2) + 3) / 4;
  p.staging_off = staging_offset(x->world, x->rows, x->head_dim);
  p.flags_off = flags_offset(x->world, x->rows, x->head_dim);
  const int64_t want = (p.n4 + kPushThreads - 1) / kPushThreads;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, device_sm_count())));
  push_kernel<<<grid, kPushThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_cuda(cudaGetLastError(), "exchange push launch");
}

int iak_exchange_merge(const iak_peer_exchange* x, void* out, int32_t out_dtype, int64_t out_row_stride,
                       uint32_t* status, uint32_t timeout_us, void* stream) {
  int st = check_exchange(x);
  if (st) return st;
  if (!out) return fail(IAK_ERR_INVALID_ARG, "out is NULL");
  if (out_dtype < 0 || out_dtype > 2) return fail(IAK_ERR_INVALID_ARG, "bad out dtype");
  if (out_row_stride < x->head_dim) return fail(IAK_ERR_INVALID_ARG, "out_row_stride < head_dim");
  if (x->rows == 0) return IAK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float* own = static_cast<const float*>(x->areas[x->rank]);
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(reinterpret_cast<const char*>(own) +
                                                           flags_offset(x->world, x->rows, x->head_dim));
  const int threads = x->head_dim >= 128 ? 128 : (x->head_dim >= 64 ? 64 : 32);
  const int64_t blocks = std::min<int64_t>(x->rows, 65535LL * 8);
  exchange_merge_kernel<<<static_cast<unsigned>(blocks), threads, x->world * sizeof(float), s>>>(
      own, flags, x->world, x->rows, x->head_dim, block_stride(x->rows, x->head_dim), out, out_dtype, out_row_stride,
      status, static_cast<uint64_t>(timeout_us) * 1000ull);
  return check_cuda(cudaGetLastError(), "exchange merge launch");
}

int iak_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(IAK_ERR_INVALID_ARG, "bad ipc alloc arguments");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return check_cuda(e, "ipc cudaMalloc");
  e = cudaMemset(*ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return check_cuda(e, "ipc handle");
  }
  return IAK_OK;
}

int iak_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(IAK_ERR_INVALID_ARG, "bad ipc open arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

int iak_ipc_close(void* ptr) {
  if (!ptr) return IAK_OK;
  return check_cuda(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
}

int iak_ipc_free(void* ptr) {
  if (!ptr) return IAK_OK;
  return check_cuda(cudaFree(ptr), "ipc cudaFree");
}

}  // extern "C"
