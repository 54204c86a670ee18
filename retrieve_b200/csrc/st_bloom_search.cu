// SilverTorch's bloom index searches on the device, the upstream-shaped st:: ops that
// evaluate query plans over the bundle-major bloom index outside st::search:
//
//  * st::bloom_index_search_batch(_prepared) (silvertorch/ops/csrc/bloom_index_search.cpp
//    :550-588; CUDA bloom_index_search_cuda.cu:1504-1640, 1832-1859): plan q over every
//    64-doc column of the index, the packed int64 word (doc 64 c + i at bit 63 - i) or 64
//    bools per column.
//  * st::generate_column_info_for_clusters (bloom_index_search.cpp:494-538): per probed
//    cluster range (start, length) its column count ceil((length + start % 64) / 64) (0 for
//    an empty range), first column start / 64 and bit offset start % 64.
//  * st::bloom_index_search_batch_return_partial_response(_prepared) (bloom_index_search.cpp
//    :244-374; CUDA bloom_index_search_cuda.cu:1780-1944): the words of only the probed
//    clusters' columns, cluster after cluster, addressed by the inclusive cumsum of the
//    column counts; row b runs plan query_plan_index[b] (or b).
//
// One thread per output word; bloom_plan_word (st_filters.cuh) is the per-column plan
// evaluation st::search's bloom filter uses, so the searches and the filter agree bit for bit.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "rb_capi_internal.h"
#include "st_filters.cuh"

namespace rb {
namespace {

constexpr int kThreads = 256;
constexpr int kScanThreads = 1024;

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int grid_for(int64_t n) {
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + kThreads - 1) / kThreads, cap)));
}

// Plan q over column c, q < plan_count, c < n_cols: the word, or 64 bytes of 0 / 1.
template <bool BOOL>
__global__ void __launch_bounds__(kThreads) bloom_search_kernel(BloomArgs a, int64_t n_cols, int64_t n_out,
                                                                void* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_out;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t q = i / n_cols, c = i % n_cols;
    const uint64_t w = bloom_plan_word(a, q, c);
    if constexpr (BOOL) {
      // byte j of the column's 64 is doc 64 c + j: bit 63 - j of the word
      uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(out) + i * 64);
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint32_t lanes[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j0 = 16 * v + 4 * u;
          lanes[u] = static_cast<uint32_t>((w >> (63 - j0)) & 1ull) |
                     static_cast<uint32_t>((w >> (62 - j0)) & 1ull) << 8 |
                     static_cast<uint32_t>((w >> (61 - j0)) & 1ull) << 16 |
                     static_cast<uint32_t>((w >> (60 - j0)) & 1ull) << 24;
        }
        dst[v] = make_uint4(lanes[0], lanes[1], lanes[2], lanes[3]);
      }
    } else {
      static_cast<uint64_t*>(out)[i] = w;
    }
  }
}

__global__ void __launch_bounds__(kThreads) column_info_kernel(const int64_t* __restrict__ offsets,
                                                               const int64_t* __restrict__ lengths, int64_t n,
                                                               int32_t* __restrict__ counts,
                                                               int32_t* __restrict__ start_cols,
                                                               int8_t* __restrict__ first) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t start = offsets[i], len = lengths[i];
    const int64_t off = start % 64;
    start_cols[i] = static_cast<int32_t>(start / 64);
    first[i] = static_cast<int8_t>(off);
    counts[i] = len > 0 ? static_cast<int32_t>((len + off + 63) / 64) : 0;
  }
}

// Inclusive cumsum of n int32 counts (int32 like the reference's cumsum(dtype=kInt)): one CTA,
// each thread a contiguous run, a block-wide scan of the run totals between two passes.
__global__ void __launch_bounds__(kScanThreads) cumsum_i32_kernel(const int32_t* __restrict__ in, int64_t n,
                                                                 int32_t* __restrict__ out) {
  __shared__ int64_t part[kScanThreads];
  const int tid = threadIdx.x;
  const int64_t per = (n + kScanThreads - 1) / kScanThreads;
  const int64_t i0 = min(n, tid * per), i1 = min(n, i0 + per);
  int64_t run = 0;
  for (int64_t i = i0; i < i1; ++i) run += in[i];
  part[tid] = run;
  __syncthreads();
  for (int off = 1; off < kScanThreads; off <<= 1) {
    const int64_t x = tid >= off ? part[tid - off] : 0;
    __syncthreads();
    part[tid] += x;
    __syncthreads();
  }
  int64_t acc = part[tid] - run;
  for (int64_t i = i0; i < i1; ++i) {
    acc += in[i];
    out[i] = static_cast<int32_t>(acc);
  }
}

// Word i < min(total, max_columns) of the partial response: the cluster range it belongs to
// (first inclusive cumsum entry above i), that range's column, the row's plan.
__global__ void __launch_bounds__(kThreads) partial_fill_kernel(BloomArgs a, const int32_t* __restrict__ cumsum,
                                                                const int32_t* __restrict__ start_cols,
                                                                int64_t n_pairs, int P, int64_t max_columns,
                                                                uint64_t* __restrict__ out) {
  const int64_t total = min(static_cast<int64_t>(cumsum[n_pairs - 1]), max_columns);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t lo = 0, hi = n_pairs - 1;  // cumsum[hi] > i
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (cumsum[mid] > i) hi = mid; else lo = mid + 1;
    }
    const int64_t before = lo == 0 ? 0 : cumsum[lo - 1];
    const int64_t row = lo / P;
    const int64_t plan = a.plan_index ? a.plan_index[row] : row;
    out[i] = bloom_plan_word(a, plan, static_cast<int64_t>(start_cols[lo]) + (i - before));
  }
}

int bloom_args(const int64_t* bloom_index, int64_t index_words, const int64_t* bundle_b_offsets, int64_t n_bundles,
               const int64_t* plans, int64_t plan_words, int plan_count, int max_stack_size, int k, int hash_k,
               const int64_t* query_plan_index, const char* who, BloomArgs& a) {
  if (bloom_index == nullptr || bundle_b_offsets == nullptr || plans == nullptr || index_words < 0 ||
      n_bundles < 0 || plan_count < 0 || plan_words < 8 * static_cast<int64_t>(plan_count) || k < 1 || hash_k < 1 ||
      max_stack_size < 0) {
    set_last_error(who);
    return RB_ERR_INVALID_ARG;
  }
  if (k > kBloomMaxK || max_stack_size > kBloomStack) {
    set_last_error("bloom search: k > 10 or a plan stack deeper than 16 is not supported");
    return RB_ERR_UNSUPPORTED;
  }
  a = BloomArgs{reinterpret_cast<const uint64_t*>(bloom_index), index_words, bundle_b_offsets, n_bundles, plans,
                plan_words, plan_count, query_plan_index, k, hash_k};
  return RB_OK;
}

}  // namespace
}  // namespace rb

using namespace rb;

extern "C" {

int rb_st_bloom_search(const int64_t* bloom_index, int64_t index_words, const int64_t* bundle_b_offsets,
                       int64_t n_bundles, const int64_t* plans, int64_t plan_words, int plan_count,
                       int max_stack_size, int k, int hash_k, int return_bool_mask, void* out, void* stream) {
  BloomArgs a;
  int rc = bloom_args(bloom_index, index_words, bundle_b_offsets, n_bundles, plans, plan_words, plan_count,
                      max_stack_size, k, hash_k, nullptr,
                      "bloom_index_search_batch: needs the index, bundle offsets, plans of plan_count slots, k and "
                      "hash_k",
                      a);
  if (rc != RB_OK) return rc;
  const int64_t n_cols = n_bundles * kBundleColumns;
  const int64_t n_out = n_cols * plan_count;
  if (n_out == 0) return RB_OK;
  if (out == nullptr) {
    set_last_error("bloom_index_search_batch: null output");
    return RB_ERR_INVALID_ARG;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (return_bool_mask)
    bloom_search_kernel<true><<<grid_for(n_out), kThreads, 0, s>>>(a, n_cols, n_out, out);
  else
    bloom_search_kernel<false><<<grid_for(n_out), kThreads, 0, s>>>(a, n_cols, n_out, out);
  return launch_status();
}

int rb_st_bloom_column_info(const int64_t* selected_cluster_offsets, const int64_t* selected_cluster_lengths,
                            int64_t n, int32_t* out_column_counts, int32_t* out_start_column_ids,
                            int8_t* out_first_item_offsets, int32_t* out_column_counts_cumsum, void* stream) {
  if (n < 0 || (n > 0 && (selected_cluster_offsets == nullptr || selected_cluster_lengths == nullptr ||
                          out_column_counts == nullptr || out_start_column_ids == nullptr ||
                          out_first_item_offsets == nullptr))) {
    set_last_error("generate_column_info_for_clusters: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  if (n == 0) return RB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  column_info_kernel<<<grid_for(n), kThreads, 0, s>>>(selected_cluster_offsets, selected_cluster_lengths, n,
                                                       out_column_counts, out_start_column_ids,
                                                       out_first_item_offsets);
  if (out_column_counts_cumsum != nullptr)
    cumsum_i32_kernel<<<1, kScanThreads, 0, s>>>(out_column_counts, n, out_column_counts_cumsum);
  return launch_status();
}

int rb_st_bloom_partial_search(const int64_t* bloom_index, int64_t index_words, const int64_t* bundle_b_offsets,
                               int64_t n_bundles, const int64_t* plans, int64_t plan_words, int plan_count,
                               int max_stack_size, const int64_t* query_plan_index, int B, int P,
                               const int32_t* column_counts_cumsum, const int32_t* start_column_ids, int k,
                               int hash_k, int64_t* out_column_mask_response, int64_t max_columns, void* stream) {
  BloomArgs a;
  int rc = bloom_args(bloom_index, index_words, bundle_b_offsets, n_bundles, plans, plan_words, plan_count,
                      max_stack_size, k, hash_k, query_plan_index,
                      "bloom_index_search_batch_return_partial_response: needs the index, bundle offsets, plans of "
                      "plan_count slots, k and hash_k",
                      a);
  if (rc != RB_OK) return rc;
  if (B < 0 || P < 0 || max_columns < 0 ||
      (static_cast<int64_t>(B) * P > 0 && (column_counts_cumsum == nullptr || start_column_ids == nullptr)) ||
      (max_columns > 0 && out_column_mask_response == nullptr)) {
    set_last_error("bloom_index_search_batch_return_partial_response: bad sizes");
    return RB_ERR_INVALID_ARG;
  }
  if (max_columns == 0) return RB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // words past the device total stay zero (the prepared form's static capacity)
  cudaError_t e = cudaMemsetAsync(out_column_mask_response, 0, static_cast<size_t>(max_columns) * 8, s);
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  const int64_t n_pairs = static_cast<int64_t>(B) * P;
  if (n_pairs == 0) return RB_OK;
  partial_fill_kernel<<<grid_for(max_columns), kThreads, 0, s>>>(
      a, column_counts_cumsum, start_column_ids, n_pairs, P, max_columns,
      reinterpret_cast<uint64_t*>(out_column_mask_response));
  return launch_status();
}

}  // extern "C"
