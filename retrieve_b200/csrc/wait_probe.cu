// rb_wait_probe: a test aid for the bounded waits every pipelined kernel here
// relies on. One CTA of the dense scan's shape (a producer warp, an MMA warp and
// epilogue warps) in which every role waits on an mbarrier that nothing ever
// completes, through the same mbar_wait the scan kernels use, with a caller-set
// limit. Each role gives up when the limit runs out (or when another role has
// raised the CTA's abort flag), records its timeout code in the workspace's
// error word, and the kernel returns: the context stays usable and the host reads
// the code with rb_workspace_device_error.
#include <cuda_runtime.h>

#include "rb_capi_internal.h"

namespace rb {

__global__ void __launch_bounds__(128, 1) wait_probe_kernel(uint64_t limit_ns, int* err) {
  __shared__ __align__(8) uint64_t never;  // a barrier with one pending arrival that never comes
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&never, 1);
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort = &abort_flag;
  // the roles of the scan kernels: producer (warp 0), MMA issuer (warp 1), epilogue (warps 2, 3)
  const int code = warp == 0 ? kDevTimeoutProducer : (warp == 1 ? kDevTimeoutMma : kDevTimeoutEpilogue);
  if (lane == 0 && !mbar_wait(&never, 0, abort, limit_ns)) {
    atomicCAS(err, 0, code);  // the first role to give up names the error
    *abort = 1;
  }
  __syncthreads();
}

}  // namespace rb

using namespace rb;

extern "C" {

int rb_wait_probe(int64_t limit_ns, void* workspace, size_t workspace_bytes, void* stream) {
  if (limit_ns < 1000 || limit_ns > 2000000000 || workspace == nullptr || workspace_bytes < 256) {
    set_last_error("wait_probe: limit_ns in [1 us, 2 s] and a workspace of at least 256 bytes");
    return RB_ERR_INVALID_ARG;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* err = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + workspace_bytes - 256);
  if (cudaMemsetAsync(err, 0, sizeof(int), s) != cudaSuccess) {
    set_last_error("wait_probe: memset failed");
    return RB_ERR_CUDA;
  }
  wait_probe_kernel<<<1, 128, 0, s>>>(static_cast<uint64_t>(limit_ns), err);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

}  // extern "C"
