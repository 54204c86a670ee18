// rb_dense_topk_noalloc: the fused dense top-k for callers that cannot
// allocate device memory on the call path.
//
// Who cannot allocate: hosts whose device memory is owned by another allocator
// and fixed at start-up (a serving process that reserves its HBM once, where a
// cudaMalloc mid-request could fail or fragment that reservation), and
// foreign-language runtimes bound through the C-ABI with no caching allocator,
// where a cudaMalloc / cudaFree pair per call would synchronise the device on
// every search. Instead of a caller-provided workspace, this entry point uses
// one file-scope device array of kNoAllocScratchBytes, reserved on every GPU
// that loads the library for the life of the process.
//
// The array's name is a host-side stand-in in host code, not a device address:
// the device address is looked up once per device with cudaGetSymbolAddress,
// on the first call made with that device current, and cached (keyed by the
// device ordinal, so a cudaDeviceReset of that device leaves the cached address
// stale: do not use this entry point on a device after resetting it). That
// first call may load the module, so it should come before any stream capture.
//
// All calls on a device share the one array and it keeps the last call's
// contents; the only word the kernels need at zero (the error word) is cleared
// by every call. Calls that overlap on the GPU (different streams, or host
// threads racing) race on the array: serialise them.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>

#include "rb_capi_internal.h"

namespace rb {

constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(32) << 20;  // 32 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
static std::atomic<void*> g_scratch_addr[kMaxDevices];

// The current device's address of g_noalloc_scratch; the stream must belong to
// that device (its scratch is the one the kernels will be given).
static int scratch_address(cudaStream_t stream, void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_last_error("dense_topk_noalloc: no usable current device");
    return RB_ERR_CUDA;
  }
  if (stream != nullptr) {
    int sdev = -1;
    if (cudaStreamGetDevice(stream, &sdev) != cudaSuccess) {
      set_last_error("dense_topk_noalloc: cannot read the stream's device");
      return RB_ERR_CUDA;
    }
    if (sdev != dev) {
      set_last_error("dense_topk_noalloc: the stream belongs to another device than the current one");
      return RB_ERR_INVALID_ARG;
    }
  }
  void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_last_error(cudaGetErrorString(e));
      return RB_ERR_CUDA;
    }
    g_scratch_addr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return RB_OK;
}

}  // namespace rb

using namespace rb;

extern "C" {

size_t rb_dense_topk_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int rb_dense_topk_noalloc(const void* queries, const void* items, int B, int N, int D, int dtype, int k,
                          int64_t id_offset, int64_t* out_ids, float* out_scores, void* stream) {
  // rb_dense_topk's argument checks, in its order and with its codes, before the size check
  if (dtype != RB_F16 && dtype != RB_BF16) {
    set_last_error("dense_topk_noalloc: dtype must be f16 or bf16");
    return RB_ERR_TYPE;
  }
  if (B < 0 || N < 0 || k < 1) {
    set_last_error("dense_topk_noalloc: bad B, N or k");
    return RB_ERR_INVALID_ARG;
  }
  if (k > 1024) {
    set_last_error("dense_topk_noalloc: k > 1024 is not supported");
    return RB_ERR_UNSUPPORTED;
  }
  const int row_bytes = dense_row_bytes(D, dtype);
  if (row_bytes != 128 && row_bytes != 256 && row_bytes != 512) {
    set_last_error("dense_topk_noalloc: rows must be 128, 256 or 512 bytes (D = 64/128/256)");
    return RB_ERR_UNSUPPORTED;
  }
  const size_t need = dense_workspace_bytes(B, N, k, row_bytes, false);
  if (need > kNoAllocScratchBytes) {
    static thread_local char msg[192];
    std::snprintf(msg, sizeof(msg),
                  "dense_topk_noalloc: this call needs %zu bytes of scratch, above the static %zu-byte array; "
                  "use rb_dense_topk with a caller workspace",
                  need, kNoAllocScratchBytes);
    set_last_error(msg);
    return RB_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  const int rc = scratch_address(static_cast<cudaStream_t>(stream), &scratch);
  if (rc != RB_OK) return rc;
  return rb_dense_topk(queries, items, B, N, D, dtype, k, id_offset, out_ids, out_scores, scratch,
                       kNoAllocScratchBytes, stream);
}

}  // extern "C"
