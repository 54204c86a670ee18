// The exchange step of the row-sharded search through the peers' memory on one
// node (NVLink / NVSwitch): instead of an NCCL all-gather, every rank pushes its
// block of the stack straight into every peer's exchange buffer with plain peer
// stores, then raises a flag in each peer's buffer; a rank reads the stack from
// its own buffer once every peer's flag for this step is up. No multicast, no
// NVLS: plain loads and stores over the peer mappings (CUDA IPC).
//
// Exchange buffer of a rank (allocated here, mapped by the peers):
//   [flags: W x 64 bytes, flag s = the last step source rank s finished pushing]
//   [slots: 2 x W x slot_bytes, parity (step & 1), then source rank]
// Steps are counted on the device (the rank's own counter, incremented by the
// push), so a captured graph replays the exchange correctly. Two parities make
// the reuse safe: a rank pushes step t + 2 into a peer's parity only after its
// own step t + 1 merge, which waited for that peer's step t + 1 flag, which the
// peer raised after its step t reads (stream order).
//
// Every wait is bounded (2 s of %globaltimer); a wait that runs out writes
// kDevTimeoutPeer to the caller's error word and the kernel returns.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "rb_capi_internal.h"

namespace rb {

namespace {

constexpr int kFlagStride = 64;  // bytes: one cache line per source rank
constexpr int kMaxPeers = 64;
constexpr int kPushThreads = 256;
constexpr int kDevTimeoutPeer = 5;  // a peer's flag did not come up in time

struct PeerArgs {
  uint8_t* bases[kMaxPeers];  // every rank's exchange buffer (this rank's own and the peers' mappings)
  int W, rank;
  int64_t slot_bytes;
};

__device__ __forceinline__ uint8_t* slot_ptr(uint8_t* base, int W, int64_t slot_bytes, int64_t parity, int src) {
  return base + static_cast<int64_t>(W) * kFlagStride + (parity * W + src) * slot_bytes;
}

__device__ __forceinline__ void store_release_sys(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int64_t load_acquire_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Copies this rank's `bytes` (16-byte aligned) into slot (parity, rank) of every
// rank's buffer; the last block to finish raises this rank's flag in every buffer
// and advances the step counter.
__global__ void __launch_bounds__(kPushThreads) peer_push_kernel(PeerArgs a, const uint4* __restrict__ src,
                                                                int64_t bytes, int64_t* step, int* done) {
  const int64_t s = *step + 1;  // the step this push completes
  const int64_t parity = s & 1;
  const int64_t n16 = bytes / 16;
  const int64_t per_dst = (n16 + gridDim.x - 1) / gridDim.x;
  const int64_t lo = blockIdx.x * per_dst, hi = min(n16, lo + per_dst);
  for (int d = 0; d < a.W; ++d) {
    uint4* dst = reinterpret_cast<uint4*>(slot_ptr(a.bases[d], a.W, a.slot_bytes, parity, a.rank));
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = src[i];
  }
  __threadfence_system();
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(done, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (last && threadIdx.x < a.W) {
    __threadfence_system();
    store_release_sys(reinterpret_cast<int64_t*>(a.bases[threadIdx.x] + a.rank * kFlagStride), s);
  }
  if (last && threadIdx.x == 0) {
    *done = 0;   // ready for the next push
    *step = s;   // read by the wait that follows on this stream
  }
}

// Waits until every rank's flag in this rank's buffer shows the current step, then
// copies the step's slots (one per source rank, in rank order) to `out`.
__global__ void __launch_bounds__(kPushThreads) peer_wait_copy_kernel(PeerArgs a, const int64_t* step, int64_t bytes,
                                                                      uint4* __restrict__ out, int* err) {
  __shared__ int ok;
  const int64_t s = *step;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x < a.W) {
    const int64_t* flag = reinterpret_cast<const int64_t*>(a.bases[a.rank] + threadIdx.x * kFlagStride);
    if (load_acquire_sys(flag) < s) {
      const uint64_t t0 = globaltimer_ns();
      while (load_acquire_sys(flag) < s) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicCAS(err, 0, kDevTimeoutPeer);
          ok = 0;
          break;
        }
        __nanosleep(200);
      }
    }
  }
  __syncthreads();
  if (!ok) return;
  const int64_t n16 = bytes / 16;
  const int64_t total = n16 * a.W;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t src_rank = i / n16, j = i - src_rank * n16;
    const uint4* slot = reinterpret_cast<const uint4*>(
        slot_ptr(a.bases[a.rank], a.W, a.slot_bytes, s & 1, static_cast<int>(src_rank)));
    out[i] = __ldcg(slot + j);  // written over NVLink by the peers: read past L1
  }
}

}  // namespace

}  // namespace rb

using namespace rb;

extern "C" {

int rb_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0) {
    set_last_error("ipc_alloc: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any peer maps it
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int rb_ipc_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) {
    set_last_error("ipc_open: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int rb_ipc_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int rb_ipc_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

size_t rb_peer_buffer_bytes(int W, int64_t slot_bytes) {
  if (W <= 0 || slot_bytes < 0) return 0;
  return static_cast<size_t>(W) * kFlagStride + static_cast<size_t>(2 * W) * static_cast<size_t>(slot_bytes);
}

int rb_peer_allgather(void* const* bases, int W, int rank, int64_t slot_bytes, const void* src, int64_t bytes,
                      int64_t* step, int* done, int* err, void* out, void* stream) {
  if (bases == nullptr || W < 1 || W > kMaxPeers || rank < 0 || rank >= W || slot_bytes <= 0 || src == nullptr ||
      bytes < 0 || bytes > slot_bytes || (bytes & 15) != 0 || (slot_bytes & 15) != 0 || step == nullptr ||
      done == nullptr || err == nullptr || out == nullptr || (reinterpret_cast<uintptr_t>(src) & 15u) != 0 ||
      (reinterpret_cast<uintptr_t>(out) & 15u) != 0) {
    set_last_error("peer_allgather: bad arguments (16-byte sizes and source, bytes <= slot_bytes, W <= 64)");
    return RB_ERR_INVALID_ARG;
  }
  PeerArgs a;
  for (int i = 0; i < W; ++i) a.bases[i] = static_cast<uint8_t*>(bases[i]);
  a.W = W;
  a.rank = rank;
  a.slot_bytes = slot_bytes;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n16 = bytes / 16;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n16 + 4095) / 4096, 132)));
  peer_push_kernel<<<blocks, kPushThreads, 0, s>>>(a, static_cast<const uint4*>(src), bytes, step, done);
  const int copy_blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n16 * W + 4095) / 4096, 132)));
  peer_wait_copy_kernel<<<copy_blocks, kPushThreads, 0, s>>>(a, step, bytes, static_cast<uint4*>(out), err);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

}  // extern "C"
