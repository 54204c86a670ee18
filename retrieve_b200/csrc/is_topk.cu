// st::is_topk on the device (silvertorch/ops/csrc/is_topk_cuda.cu:83-149): per row b of
// scores [B, n] the value at position clamp(ks[b] - 1, 0, n - 1) of the row sorted descending
// (ascending with largest = false; NaN sorts as the largest value either way), then
// out[b, j] = (scores[b, j] >= kth) (<= for smallest), compared in fp32 and written as 1 / 0 in
// the scores' type. The reference sorts every row; here one CTA per row finds the kth value by
// an exact 4-pass radix select over order-preserving 32-bit keys (NaN the largest key) and writes
// the row's flags.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "rb_capi_internal.h"
#include "rb_common.cuh"

namespace rb {
namespace {

constexpr int kThreads = 512;

template <typename T>
__device__ __forceinline__ float load_f32(const T* p, int64_t i);
template <>
__device__ __forceinline__ float load_f32<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float load_f32<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }
template <>
__device__ __forceinline__ float load_f32<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Order-preserving key of a float: larger value, larger key; every NaN the largest key.
__device__ __forceinline__ uint32_t sort_key(float v) { return v != v ? 0xffffffffu : f2ord(v); }

template <typename T>
__global__ void __launch_bounds__(kThreads) is_topk_kernel(const T* __restrict__ scores, int64_t n,
                                                           const int64_t* __restrict__ ks, bool largest,
                                                           T* __restrict__ out) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_rank;
  const int64_t b = blockIdx.x;
  const T* row = scores + b * n;
  int64_t kk = ks[b] - 1;
  kk = kk < 0 ? 0 : (kk > n - 1 ? n - 1 : kk);
  // rank of the wanted element in descending key order
  const int64_t rank = largest ? kk : n - 1 - kk;
  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_rank = static_cast<uint32_t>(rank);
  }
  uint32_t mask = 0;  // key bits fixed so far
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
      const uint32_t key = sort_key(load_f32(row, j));
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xffu], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t r = s_rank;
      int digit = 255;
      for (; digit > 0; --digit) {  // from the largest digit down
        if (r < hist[digit]) break;
        r -= hist[digit];
      }
      s_prefix = prefix | (static_cast<uint32_t>(digit) << shift);
      s_rank = r;
    }
    mask |= 0xffu << shift;
    __syncthreads();
  }
  const uint32_t kth_key = s_prefix;
  const float kth = kth_key == 0xffffffffu ? __int_as_float(0x7fc00000) : ord2f(kth_key);
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
    const float v = load_f32(row, j);
    const bool sel = largest ? (v >= kth) : (v <= kth);
    out[b * n + j] = from_f32<T>(sel ? 1.0f : 0.0f);
  }
}

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

}  // namespace
}  // namespace rb

using namespace rb;

extern "C" {

int rb_st_is_topk(const void* scores, int dtype, int64_t B, int64_t n, const int64_t* ks, int largest, void* out,
                  void* stream) {
  if (B < 0 || n < 0 || B > INT32_MAX || n > UINT32_MAX ||
      (B > 0 && n > 0 && (scores == nullptr || ks == nullptr || out == nullptr))) {
    set_last_error("is_topk: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  if (dtype != RB_F32 && dtype != RB_F16 && dtype != RB_BF16) {
    set_last_error("is_topk: scores must be fp32, fp16 or bf16");
    return RB_ERR_TYPE;
  }
  if (B == 0 || n == 0) return RB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>(B);
  if (dtype == RB_F32)
    is_topk_kernel<float><<<grid, kThreads, 0, s>>>(static_cast<const float*>(scores), n, ks, largest != 0,
                                                    static_cast<float*>(out));
  else if (dtype == RB_F16)
    is_topk_kernel<__half><<<grid, kThreads, 0, s>>>(static_cast<const __half*>(scores), n, ks, largest != 0,
                                                     static_cast<__half*>(out));
  else
    is_topk_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(scores), n, ks,
                                                            largest != 0, static_cast<__nv_bfloat16*>(out));
  return launch_status();
}

}  // extern "C"
