// st::take_top_k_and_gather_from_main_and_fresh on the device
// (silvertorch/ops/csrc/fresh_index_post_processing.cpp:226-272; its gather :33-128): per row the
// top min(k, Mf + Mm) of the fresh scores followed by the main scores (the merged column j < Mf is
// fresh column j, else main column j - Mf), largest first — NaN the largest, as torch.topk
// ranks it; ties, which torch.topk leaves unordered, to the lower merged column — then, per data
// key, the rows the winners point at: fresh_data[fresh_indices[b, j]] for a fresh winner,
// main_data[main_indices[b, j - Mf]] for a main one, row 0 when that index is outside the table.
//
//  fresh_topk_kernel: one CTA per row sorts the row's Mf + Mm 64-bit keys (order-preserving score
//    key above, the complement of the merged column below) with a bitonic sort in shared memory
//    (Mf + Mm <= 4096) and writes the first k'.
//  fresh_gather_kernel: one thread per output element copies it from its source row.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "rb_capi_internal.h"
#include "rb_common.cuh"

namespace rb {
namespace {

constexpr int kThreads = 512;
constexpr int kMaxMerged = 4096;

__device__ __forceinline__ float score_at(const void* p, int dtype, int64_t i) {
  if (dtype == RB_F32) return static_cast<const float*>(p)[i];
  if (dtype == RB_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void copy_score(const void* src, int64_t si, void* dst, int64_t di, int dtype) {
  if (dtype == RB_F32)
    static_cast<float*>(dst)[di] = static_cast<const float*>(src)[si];
  else
    static_cast<uint16_t*>(dst)[di] = static_cast<const uint16_t*>(src)[si];
}

__global__ void __launch_bounds__(kThreads) fresh_topk_kernel(const void* __restrict__ fresh, int64_t mf,
                                                              const void* __restrict__ main_, int64_t mm, int dtype,
                                                              int kk, int m_pow2, void* __restrict__ out_scores,
                                                              int64_t* __restrict__ out_idx,
                                                              uint8_t* __restrict__ out_fresh) {
  extern __shared__ __align__(16) uint64_t keys[];
  const int64_t b = blockIdx.x;
  const int64_t m = mf + mm;
  for (int i = threadIdx.x; i < m_pow2; i += blockDim.x) {
    uint64_t key = 0;  // padding sorts last: every real key is above it
    if (i < m) {
      const float v = i < mf ? score_at(fresh, dtype, b * mf + i) : score_at(main_, dtype, b * mm + (i - mf));
      const uint32_t sk = v != v ? 0xffffffffu : f2ord(v);
      key = (static_cast<uint64_t>(sk) << 32) | (0xffffffffu - static_cast<uint32_t>(i));
    }
    keys[i] = key;
  }
  __syncthreads();
  // bitonic sort, descending
  for (int size = 2; size <= m_pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < m_pow2; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const uint64_t a = keys[i], c = keys[j];
          if (desc ? (a < c) : (a > c)) {
            keys[i] = c;
            keys[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int j = threadIdx.x; j < kk; j += blockDim.x) {
    const int64_t col = static_cast<int64_t>(0xffffffffu - static_cast<uint32_t>(keys[j] & 0xffffffffu));
    const int64_t o = b * kk + j;
    out_idx[o] = col;
    out_fresh[o] = col < mf ? 1 : 0;
    if (col < mf)
      copy_score(fresh, b * mf + col, out_scores, o, dtype);
    else
      copy_score(main_, b * mm + (col - mf), out_scores, o, dtype);
  }
}

__device__ __forceinline__ int64_t index_at(const void* p, bool i64, int64_t i) {
  return i64 ? static_cast<const int64_t*>(p)[i] : static_cast<const int32_t*>(p)[i];
}

__global__ void fresh_gather_kernel(const int64_t* __restrict__ top_idx, int64_t n_out, int kk, int64_t mf,
                                    int64_t mm, const void* __restrict__ fresh_idx, const void* __restrict__ main_idx,
                                    bool idx64, const uint8_t* __restrict__ fresh_data, int64_t fresh_rows,
                                    const uint8_t* __restrict__ main_data, int64_t main_rows, int64_t row_elems,
                                    int elem_bytes, uint8_t* __restrict__ out) {
  const int64_t total = n_out * row_elems;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t o = t / row_elems, e = t - o * row_elems;
    const int64_t b = o / kk;
    const int64_t col = top_idx[o];
    const uint8_t* src;
    int64_t row;
    if (col < mf) {
      row = index_at(fresh_idx, idx64, b * mf + col);
      if (row < 0 || row >= fresh_rows) row = 0;
      src = fresh_data;
    } else {
      row = index_at(main_idx, idx64, b * mm + (col - mf));
      if (row < 0 || row >= main_rows) row = 0;
      src = main_data;
    }
    const uint8_t* s = src + (row * row_elems + e) * elem_bytes;
    uint8_t* d = out + t * elem_bytes;
    for (int i = 0; i < elem_bytes; ++i) d[i] = s[i];
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

int rb_st_fresh_topk(const void* fresh_scores, int64_t mf, const void* main_scores, int64_t mm, int dtype,
                     int64_t B, int k, void* out_scores, int64_t* out_idx, uint8_t* out_is_fresh, void* stream) {
  if (B < 0 || mf < 0 || mm < 0 || k < 0 || B > INT32_MAX) {
    set_last_error("take_top_k_and_gather_from_main_and_fresh: bad sizes");
    return RB_ERR_INVALID_ARG;
  }
  if (dtype != RB_F32 && dtype != RB_F16 && dtype != RB_BF16) {
    set_last_error("take_top_k_and_gather_from_main_and_fresh: scores must be fp32, fp16 or bf16");
    return RB_ERR_TYPE;
  }
  const int64_t m = mf + mm;
  if (m > kMaxMerged) {
    set_last_error("take_top_k_and_gather_from_main_and_fresh: more than 4096 fresh + main columns");
    return RB_ERR_UNSUPPORTED;
  }
  const int kk = static_cast<int>(k < m ? k : m);
  if (B == 0 || kk == 0) return RB_OK;
  if ((mf > 0 && fresh_scores == nullptr) || (mm > 0 && main_scores == nullptr) || out_scores == nullptr ||
      out_idx == nullptr || out_is_fresh == nullptr) {
    set_last_error("take_top_k_and_gather_from_main_and_fresh: null tensor");
    return RB_ERR_INVALID_ARG;
  }
  int m_pow2 = 1;
  while (m_pow2 < m) m_pow2 <<= 1;
  fresh_topk_kernel<<<static_cast<unsigned>(B), kThreads, static_cast<size_t>(m_pow2) * 8,
                      static_cast<cudaStream_t>(stream)>>>(fresh_scores, mf, main_scores, mm, dtype, kk, m_pow2,
                                                           out_scores, out_idx, out_is_fresh);
  return launch_status();
}

int rb_st_fresh_gather(const int64_t* top_idx, int64_t B, int k_out, int64_t mf, int64_t mm,
                       const void* fresh_indices, const void* main_indices, int indices_are_int64,
                       const void* fresh_data, int64_t fresh_rows, const void* main_data, int64_t main_rows,
                       int64_t row_elems, int elem_bytes, void* out, void* stream) {
  if (B < 0 || k_out < 0 || mf < 0 || mm < 0 || fresh_rows < 0 || main_rows < 0 || row_elems < 0 ||
      (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)) {
    set_last_error("take_top_k_and_gather_from_main_and_fresh: bad gather sizes");
    return RB_ERR_INVALID_ARG;
  }
  const int64_t n_out = B * k_out;
  if (n_out == 0 || row_elems == 0) return RB_OK;
  // a table without rows has no row 0 to fall back to
  if (top_idx == nullptr || out == nullptr || (mf > 0 && (fresh_indices == nullptr || fresh_rows == 0)) ||
      (mm > 0 && (main_indices == nullptr || main_rows == 0))) {
    set_last_error("take_top_k_and_gather_from_main_and_fresh: a source with winners has no rows");
    return RB_ERR_INVALID_ARG;
  }
  const int64_t total = n_out * row_elems;
  const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
  fresh_gather_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      top_idx, n_out, k_out, mf, mm, fresh_indices, main_indices, indices_are_int64 != 0,
      static_cast<const uint8_t*>(fresh_data), fresh_rows, static_cast<const uint8_t*>(main_data), main_rows,
      row_elems, elem_bytes, static_cast<uint8_t*>(out));
  return launch_status();
}

}  // extern "C"
