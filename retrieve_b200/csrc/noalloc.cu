// rb_dense_topk_noalloc: the fused dense top-k for callers that cannot
// allocate device memory on the call path.
//
// Who cannot allocate: a host that records the search into a CUDA graph
// (cudaMalloc is not permitted while a stream is being captured), and hosts
// whose device memory is owned by another allocator and fixed at start-up (a
// serving process that pre-reserves HBM, or a foreign-language runtime bound
// through the C-ABI with no caching allocator, where a cudaMalloc per call
// would synchronise the device and could fail mid-request). Instead of a
// caller-provided workspace, this entry point uses one file-scope device array
// of kNoAllocScratchBytes, reserved on every GPU that loads the library for the
// life of the process.
//
// The array's name is a host-side stand-in in host code, not a device address:
// the device address is looked up once per device with cudaGetSymbolAddress,
// on the first call made with that device current, and cached. That first call
// may load the module, so it should come before any stream capture.
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

static int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_last_error("dense_topk_noalloc: no usable current device");
    return RB_ERR_CUDA;
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
  if (B < 0 || N < 0 || k < 1) {
    set_last_error("dense_topk_noalloc: bad B, N or k");
    return RB_ERR_INVALID_ARG;
  }
  const size_t need = dense_workspace_bytes(B, N, k, dense_row_bytes(D, dtype), dense_scaled(dtype));
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
  const int rc = scratch_address(&scratch);
  if (rc != RB_OK) return rc;
  return rb_dense_topk(queries, items, B, N, D, dtype, k, id_offset, out_ids, out_scores, scratch,
                       kNoAllocScratchBytes, stream);
}

}  // extern "C"
