// Per-query merge of candidate lists into the final top-k: one 256-thread CTA
// per query runs an exact radix select over the concatenated lists (composite
// key: score descending, then id ascending), sorts the k winners with a bitonic
// network in shared memory and writes (ids int64, scores fp32), padding rows
// with fewer than k candidates with -1 / -inf (functional.py:57-85 `masked_topk`
// pad_to_k semantics). The k-th score is also written out: it seeds the
// threshold of the next scan pass.
#include <algorithm>
#include <cstdint>

#include "rb_capi_internal.h"
#include "rb_common.cuh"
#include "rb_select.cuh"

namespace rb {

constexpr int kMaxK = 1024;

__global__ void __launch_bounds__(kMergeThreads) merge_lists_kernel(const uint2* __restrict__ lists,
                                                                    const int* __restrict__ counts, int n_lists,
                                                                    int stride, int k, int64_t id_offset,
                                                                    int64_t* __restrict__ out_ids,
                                                                    float* __restrict__ out_scores,
                                                                    float* __restrict__ out_kth) {
  __shared__ MergeSmem sm;
  __shared__ uint64_t keys[kMaxK];
  const int q = blockIdx.x;
  const int tid = threadIdx.x;
  ListSet ls{lists + static_cast<size_t>(q) * n_lists * stride, counts + static_cast<size_t>(q) * n_lists, n_lists,
             stride};
  int total = 0;
  for (int r = 0; r < n_lists; ++r) total += ls.counts[r];
  const uint64_t cut = block_radix_cut(ls, total, k, sm);
  if (tid == 0) sm.n_out = 0;
  __syncthreads();
  for (int r = 0; r < n_lists; ++r) {
    const int c = ls.counts[r];
    const uint2* l = ls.base + static_cast<size_t>(r) * stride;
    for (int i = tid; i < c; i += kMergeThreads) {
      const uint2 v = l[i];
      const uint64_t key = make_key(v.x, v.y);
      if (key >= cut) {
        const uint32_t slot = atomicAdd(&sm.n_out, 1u);
        if (slot < kMaxK) keys[slot] = key;
      }
    }
  }
  __syncthreads();
  const int n_out = min(static_cast<int>(sm.n_out), k);
  int n_pad = 1;
  while (n_pad < n_out) n_pad <<= 1;
  for (int i = n_out + tid; i < n_pad; i += kMergeThreads) keys[i] = 0;
  __syncthreads();
  // bitonic sort, descending
  for (int size = 2; size <= n_pad; size <<= 1) {
    for (int st = size >> 1; st > 0; st >>= 1) {
      for (int i = tid; i < n_pad / 2; i += kMergeThreads) {
        const int lo = 2 * st * (i / st) + (i % st);
        const int hi = lo + st;
        const bool desc = (lo & size) == 0;
        const uint64_t a = keys[lo], b = keys[hi];
        if ((a < b) == desc) {
          keys[lo] = b;
          keys[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  if (out_ids != nullptr) {
    for (int i = tid; i < k; i += kMergeThreads) {
      int64_t id = -1;
      float s = -INFINITY;
      if (i < n_out) {
        const uint2 e = key_to_entry(keys[i]);
        id = static_cast<int64_t>(e.y) + id_offset;
        s = __uint_as_float(e.x);
      }
      out_ids[static_cast<size_t>(q) * k + i] = id;
      out_scores[static_cast<size_t>(q) * k + i] = s;
    }
  }
  if (out_kth != nullptr && tid == 0) {
    out_kth[q] = (n_out >= k) ? __uint_as_float(key_to_entry(keys[k - 1]).x) : -INFINITY;
  }
}

__global__ void fill_empty_kernel(int64_t* out_ids, float* out_scores, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    out_ids[i] = -1;
    out_scores[i] = -INFINITY;
  }
}

int merge_lists(const uint2* lists, const int* counts, int B, int n_lists, int stride, int k, int64_t id_offset,
                int64_t* out_ids, float* out_scores, float* out_kth, cudaStream_t stream) {
  if (k < 1 || k > kMaxK) {
    set_last_error("merge: k must be in [1, 1024]");
    return RB_ERR_INVALID_ARG;
  }
  if (B == 0) return RB_OK;
  merge_lists_kernel<<<B, kMergeThreads, 0, stream>>>(lists, counts, n_lists, stride, k, id_offset, out_ids,
                                                      out_scores, out_kth);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

// Packs W per-shard top-k lists [W, B, kin] (id -1 = empty slot) into the
// per-query candidate lists merge_lists_kernel reads: lists[b][w] of kin entries.
__global__ void pack_shard_lists_kernel(const int64_t* __restrict__ ids, const float* __restrict__ scores, int W,
                                        int B, int kin, uint2* __restrict__ lists, int* __restrict__ counts) {
  const size_t total = static_cast<size_t>(W) * B * kin;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int w = static_cast<int>(i / (static_cast<size_t>(B) * kin));
    const int b = static_cast<int>((i / kin) % B);
    const int64_t id = ids[i];
    if (id >= 0) {
      const size_t lst = static_cast<size_t>(b) * W + w;
      const int slot = atomicAdd(&counts[lst], 1);
      lists[lst * kin + slot] = make_uint2(__float_as_uint(scores[i]), static_cast<uint32_t>(id));
    }
  }
}

int merge_shard_lists(const int64_t* ids, const float* scores, int W, int B, int kin, int k, int64_t* out_ids,
                      float* out_scores, void* ws, cudaStream_t stream) {
  uint2* lists = static_cast<uint2*>(ws);
  int* counts = reinterpret_cast<int*>(static_cast<uint8_t*>(ws) +
                                       align_up(static_cast<size_t>(W) * B * kin * sizeof(uint2), 256));
  if (cudaMemsetAsync(counts, 0, static_cast<size_t>(W) * B * sizeof(int), stream) != cudaSuccess) {
    set_last_error("memset failed");
    return RB_ERR_CUDA;
  }
  const size_t total = static_cast<size_t>(W) * B * kin;
  const int blocks = static_cast<int>(std::min<size_t>((total + 255) / 256, 4096));
  if (total > 0) pack_shard_lists_kernel<<<blocks, 256, 0, stream>>>(ids, scores, W, B, kin, lists, counts);
  return merge_lists(lists, counts, B, W, kin, k, 0, out_ids, out_scores, nullptr, stream);
}

size_t merge_shard_ws_bytes(int W, int B, int kin) {
  return align_up(static_cast<size_t>(W) * B * kin * sizeof(uint2), 256) +
         align_up(static_cast<size_t>(W) * B * sizeof(int), 256);
}

void fill_empty(int64_t* out_ids, float* out_scores, size_t n, cudaStream_t stream) {
  if (n == 0) return;
  const int blocks = static_cast<int>(std::min<size_t>((n + 255) / 256, 1024));
  fill_empty_kernel<<<blocks, 256, 0, stream>>>(out_ids, out_scores, n);
}

}  // namespace rb
