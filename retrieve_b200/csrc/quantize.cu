// Per-row symmetric int8 quantization of a query batch, the query side of the
// int8 paths (retrieve/src/retrieve/indexing/quantize.py:9-18 `quantize_int8`):
//   abs_max = max(max_d |x[b, d]|, 1e-8)        (fp32)
//   scale   = abs_max * fp32(1/127)              (fp32 multiply)
//   code    = clamp(round_half_even(fp32(fp64(x) / fp64(abs_max)) * 127), -128, 127)
// The scale is what `abs_max / 127.0` gives on a CUDA tensor: torch evaluates a division by a
// CPU scalar on the device as a multiply by the scalar's fp32 reciprocal, and SilverTorch's
// query prep writes the same product (silvertorch/ops/csrc/fork_search_cuda.cu:686; the
// reference checks the two equal, retrieve/tests/parity/test_official.py:676-697). On a CPU
// tensor torch divides, which differs in the last bit for a few rows in a hundred.
// One warp per row.
#include <algorithm>
#include <cstdint>

#include "rb_capi_internal.h"
#include "rb_common.cuh"

namespace rb {

__global__ void quantize_int8_rows_kernel(const float* __restrict__ x, int B, int D, int8_t* __restrict__ codes,
                                          float* __restrict__ scales) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= B) return;
  const float* xr = x + static_cast<size_t>(row) * D;
  float m = 0.f;
  for (int d = lane; d < D; d += 32) m = fmaxf(m, fabsf(xr[d]));
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(RB_FULL_MASK, m, off));
  const float abs_max = fmaxf(m, 1e-8f);
  const double am = static_cast<double>(abs_max);
  int8_t* cr = codes + static_cast<size_t>(row) * D;
  for (int d = lane; d < D; d += 32) {
    const float r = __double2float_rn(static_cast<double>(xr[d]) / am);
    float c = rintf(__fmul_rn(r, 127.f));
    c = fminf(fmaxf(c, -128.f), 127.f);
    cr[d] = static_cast<int8_t>(c);
  }
  if (lane == 0) scales[row] = __fmul_rn(abs_max, 1.0f / 127.0f);
}

}  // namespace rb

using namespace rb;

extern "C" int rb_quantize_int8(const float* x, int B, int D, int8_t* codes, float* scales, void* stream) {
  if (B < 0 || D <= 0) {
    set_last_error("quantize_int8: bad sizes");
    return RB_ERR_INVALID_ARG;
  }
  if (B == 0) return RB_OK;
  const int warps = 8;
  quantize_int8_rows_kernel<<<(B + warps - 1) / warps, 32 * warps, 0, static_cast<cudaStream_t>(stream)>>>(
      x, B, D, codes, scales);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}
