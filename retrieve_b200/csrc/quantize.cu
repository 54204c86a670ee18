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
// A NaN in a row makes its abs_max and scale NaN and its codes 0, as torch's
// amax propagates NaN and a NaN converts to the integer 0. One warp per row.
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
  bool nan = false;
  for (int d = lane; d < D; d += 32) {
    const float a = fabsf(xr[d]);
    nan |= (a != a);
    m = fmaxf(m, a);
  }
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(RB_FULL_MASK, m, off));
  // torch's amax propagates NaN (fmaxf would drop it); a NaN code converts to 0
  nan = __any_sync(RB_FULL_MASK, nan);
  const float abs_max = nan ? __uint_as_float(0x7fc00000u) : fmaxf(m, 1e-8f);
  const double am = static_cast<double>(abs_max);
  int8_t* cr = codes + static_cast<size_t>(row) * D;
  for (int d = lane; d < D; d += 32) {
    const float r = __double2float_rn(static_cast<double>(xr[d]) / am);
    float c = rintf(__fmul_rn(r, 127.f));
    c = (c != c) ? 0.f : fminf(fmaxf(c, -128.f), 127.f);
    cr[d] = static_cast<int8_t>(c);
  }
  if (lane == 0) scales[row] = __fmul_rn(abs_max, 1.0f / 127.0f);
}

// Per-tensor symmetric int8 quantization, the item side of SilverTorch's int8
// table (retrieve/src/retrieve/indexing/quantize.py:34-52 `quantize_int8_global`,
// as it evaluates on CUDA tensors):
//   abs_max = max(max |x|, 1e-8) over the whole [N, D] table   (NaN propagates)
//   code    = clamp(round_half_even(fp32(x / abs_max) * 127), -128, 127)
//   scale   = abs_max * fp32(1/127)   (a 0-dim CUDA tensor divided by a CPU scalar)
// Pass 1 folds |x| into one word by atomicMax on the fp32 bits (non-negative
// floats order as unsigned integers, and a NaN's bits sit above +inf's); pass 2
// writes the codes of rows[i] (or of row i) into output row i.
__global__ void abs_max_kernel(const float* __restrict__ x, int64_t n, unsigned int* __restrict__ out) {
  float m = 0.f;
  bool nan = false;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float a = fabsf(x[i]);
    nan |= (a != a);
    m = fmaxf(m, a);
  }
  unsigned int bits = nan ? 0x7fc00000u : __float_as_uint(m);
  for (int off = 16; off > 0; off >>= 1) bits = max(bits, __shfl_xor_sync(RB_FULL_MASK, bits, off));
  if ((threadIdx.x & 31) == 0) atomicMax(out, bits);
}

__global__ void quantize_global_codes_kernel(const float* __restrict__ x, int64_t N, int D,
                                             const int64_t* __restrict__ rows, int64_t n_rows,
                                             const unsigned int* __restrict__ abs_max_bits, int8_t* __restrict__ codes,
                                             float* __restrict__ scale) {
  const float am_raw = __uint_as_float(*abs_max_bits);
  const float am = (am_raw != am_raw) ? am_raw : fmaxf(am_raw, 1e-8f);
  const int64_t n = n_rows * D;
  const int64_t first = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (first == 0) *scale = __fmul_rn(am, 1.0f / 127.0f);
  for (int64_t i = first; i < n; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / D;
    const int64_t src = rows ? rows[r] : r;
    int8_t c = 0;
    if (src >= 0 && src < N) {
      float v = rintf(__fmul_rn(__fdiv_rn(x[src * D + (i - r * D)], am), 127.f));
      v = (v != v) ? 0.f : fminf(fmaxf(v, -128.f), 127.f);
      c = static_cast<int8_t>(v);
    }
    codes[i] = c;
  }
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

extern "C" int rb_quantize_int8_global_workspace_size(size_t* bytes) {
  if (bytes == nullptr) {
    set_last_error("quantize_int8_global_workspace_size: null pointer");
    return RB_ERR_INVALID_ARG;
  }
  *bytes = 256;
  return RB_OK;
}

extern "C" int rb_quantize_int8_global(const float* x, int64_t N, int D, const int64_t* rows, int64_t n_rows,
                                       int8_t* codes, float* scale, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  if (N < 0 || D <= 0 || (rows != nullptr && n_rows < 0)) {
    set_last_error("quantize_int8_global: bad sizes");
    return RB_ERR_INVALID_ARG;
  }
  if (workspace == nullptr || workspace_bytes < sizeof(unsigned int)) {
    set_last_error("quantize_int8_global: workspace too small");
    return RB_ERR_WORKSPACE;
  }
  if (rows == nullptr) n_rows = N;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int* am = static_cast<unsigned int*>(workspace);
  cudaMemsetAsync(am, 0, sizeof(unsigned int), s);
  const int64_t n = N * static_cast<int64_t>(D);
  if (n > 0) {
    const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 8));
    abs_max_kernel<<<blocks, 256, 0, s>>>(x, n, am);
  }
  const int64_t m = n_rows * static_cast<int64_t>(D);
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((m + 255) / 256, 148 * 16)));
  quantize_global_codes_kernel<<<blocks, 256, 0, s>>>(x, N, D, rows, n_rows, am, codes, scale);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}
