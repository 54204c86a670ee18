// Selection kernels that run after a scan:
//
//  * merge_lists_kernel: per query, the exact top-k over its candidate lists
//    (composite key: score descending, then id ascending), written sorted as
//    (ids int64, scores fp32) and padded with -1 / -inf
//    (retrieve/src/retrieve/functional.py:57-85 `masked_topk`, pad_to_k). One
//    256-thread CTA per query: one pass over the lists histograms the top 11
//    key bits; when the bucket that holds the k-th key and everything above it
//    fit in shared memory (the usual case) they are gathered there and the rest
//    of the radix select runs on-chip; otherwise it continues over the lists.
//  * row_kth_kernel: per row of a float matrix, a lower bound on the k-th
//    largest value (the threshold seed of the full scan pass).
//  * pack_shard_lists_kernel: the multi-GPU merge input (per-rank top-k lists).
#include <algorithm>
#include <cstdint>

#include "rb_capi_internal.h"
#include "rb_common.cuh"
#include "rb_select.cuh"

namespace rb {

constexpr int kMaxK = 1024;
constexpr int kSmemKeys = 2048;
constexpr int kBins = 2048;

struct SelectShared {
  uint32_t hist[kBins];
  uint32_t warp_tot[kMergeThreads / 32];
  uint32_t digit, above, in_digit;
  uint32_t n_keys, n_out;
  uint64_t keys[kSmemKeys];
  uint64_t out[kMaxK];
};

// Finds the digit whose bucket holds the need-th largest element of a
// histogram with nbins = 256 * BPT bins. Thread t owns bins
// [nbins - BPT*(t+1), nbins - BPT*t), so a prefix over threads is a suffix over
// bins. Results land in sh.digit / sh.above / sh.in_digit.
template <int BPT>
__device__ __forceinline__ void block_find_digit_n(SelectShared& sh, uint32_t need) {
  constexpr int nbins = kMergeThreads * BPT;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t b[BPT];
  uint32_t mine = 0;
#pragma unroll
  for (int j = 0; j < BPT; ++j) {
    b[j] = sh.hist[nbins - BPT * (tid + 1) + j];  // b[BPT-1] is this thread's highest bin
    mine += b[j];
  }
  uint32_t incl = mine;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t v = __shfl_up_sync(RB_FULL_MASK, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) sh.warp_tot[warp] = incl;
  __syncthreads();
  uint32_t base = 0;
  for (int w = 0; w < warp; ++w) base += sh.warp_tot[w];
  incl += base;
  uint32_t acc = incl - mine;
  if (acc < need && need <= incl) {
#pragma unroll
    for (int j = BPT - 1; j >= 0; --j) {
      if (acc + b[j] >= need) {
        sh.digit = nbins - BPT * (tid + 1) + j;
        sh.above = acc;
        sh.in_digit = b[j];
        break;
      }
      acc += b[j];
    }
  }
  __syncthreads();
}

// Radix select with 11-bit digits (the last one 9 bits) over 64-bit keys that
// `visit` enumerates (each thread visits a strided share). Returns the cut:
// exactly k keys are >= cut. Requires total > k.
template <class Visit>
__device__ uint64_t block_radix_cut11(const Visit& visit, int k, SelectShared& sh) {
  uint64_t prefix = 0, mask = 0;
  uint32_t need = static_cast<uint32_t>(k);
  for (int shift = 53; shift >= 0; shift = (shift == 9) ? 0 : shift - 11) {
    if (shift == 0 && mask == ~0ull) break;
    const int bits = (shift == 0) ? 9 : 11;
    const uint64_t dmask = (1ull << bits) - 1;
    for (int i = threadIdx.x; i < kBins; i += kMergeThreads) sh.hist[i] = 0;
    __syncthreads();
    visit([&](uint64_t key) {
      if ((key & mask) == prefix) atomicAdd(&sh.hist[(key >> shift) & dmask], 1u);
    });
    __syncthreads();
    if (bits == 11)
      block_find_digit_n<kBins / kMergeThreads>(sh, need);
    else
      block_find_digit_n<512 / kMergeThreads>(sh, need);
    prefix |= static_cast<uint64_t>(sh.digit) << shift;
    mask |= dmask << shift;
    need -= sh.above;
    const bool done = (sh.in_digit == need);
    __syncthreads();
    if (done || shift == 0) break;
  }
  return prefix;
}

// Sorts sh.out[0, n) descending (bitonic, padded with zero keys to a power of two).
__device__ void block_sort_out(SelectShared& sh, int n) {
  const int tid = threadIdx.x;
  int n_pad = 1;
  while (n_pad < n) n_pad <<= 1;
  for (int i = n + tid; i < n_pad; i += kMergeThreads) sh.out[i] = 0;
  __syncthreads();
  for (int size = 2; size <= n_pad; size <<= 1) {
    for (int st = size >> 1; st > 0; st >>= 1) {
      for (int i = tid; i < n_pad / 2; i += kMergeThreads) {
        const int lo = 2 * st * (i / st) + (i % st);
        const int hi = lo + st;
        const bool desc = (lo & size) == 0;
        const uint64_t a = sh.out[lo], b = sh.out[hi];
        if ((a < b) == desc) {
          sh.out[lo] = b;
          sh.out[hi] = a;
        }
      }
      __syncthreads();
    }
  }
}

__global__ void __launch_bounds__(kMergeThreads) merge_lists_kernel(const uint2* __restrict__ lists,
                                                                    const int* __restrict__ counts, int n_lists,
                                                                    int stride, int k, int64_t id_offset,
                                                                    int64_t* __restrict__ out_ids,
                                                                    float* __restrict__ out_scores) {
  __shared__ SelectShared sh;
  const int q = blockIdx.x;
  const int tid = threadIdx.x;
  const uint2* qlists = lists + static_cast<size_t>(q) * n_lists * stride;
  const int* qcounts = counts + static_cast<size_t>(q) * n_lists;
  auto visit_global = [&](auto&& f) {
    for (int r = 0; r < n_lists; ++r) {
      const int c = qcounts[r];
      const uint2* l = qlists + static_cast<size_t>(r) * stride;
      for (int i = tid; i < c; i += kMergeThreads) {
        const uint2 v = l[i];
        f(make_key(v.x, v.y));
      }
    }
  };
  int total = 0;
  for (int r = 0; r < n_lists; ++r) total += qcounts[r];
  if (tid == 0) {
    sh.n_keys = 0;
    sh.n_out = 0;
  }
  __syncthreads();

  // 1) gather into shared memory: everything, or the buckets >= the k-th's
  bool on_chip = true;
  if (total <= kSmemKeys) {
    visit_global([&](uint64_t key) { sh.keys[atomicAdd(&sh.n_keys, 1u)] = key; });
  } else {
    for (int i = tid; i < kBins; i += kMergeThreads) sh.hist[i] = 0;
    __syncthreads();
    visit_global([&](uint64_t key) { atomicAdd(&sh.hist[key >> 53], 1u); });
    __syncthreads();
    block_find_digit_n<kBins / kMergeThreads>(sh, static_cast<uint32_t>(k));
    const uint32_t sel = sh.above + sh.in_digit;
    const uint64_t lo = static_cast<uint64_t>(sh.digit) << 53;
    if (sel <= static_cast<uint32_t>(kSmemKeys)) {
      visit_global([&](uint64_t key) {
        if (key >= lo) sh.keys[atomicAdd(&sh.n_keys, 1u)] = key;
      });
    } else {
      on_chip = false;
    }
  }
  __syncthreads();

  // 2) exact cut, 3) the <= k winners into sh.out
  if (on_chip) {
    const int n = static_cast<int>(sh.n_keys);
    auto visit_smem = [&](auto&& f) {
      for (int i = tid; i < n; i += kMergeThreads) f(sh.keys[i]);
    };
    const uint64_t cut = (n > k) ? block_radix_cut11(visit_smem, k, sh) : 0ull;
    for (int i = tid; i < n; i += kMergeThreads)
      if (sh.keys[i] >= cut) sh.out[atomicAdd(&sh.n_out, 1u)] = sh.keys[i];
  } else {
    const uint64_t cut = block_radix_cut11(visit_global, k, sh);
    visit_global([&](uint64_t key) {
      if (key >= cut) sh.out[atomicAdd(&sh.n_out, 1u)] = key;
    });
  }
  __syncthreads();
  const int n_out = min(static_cast<int>(sh.n_out), k);
  block_sort_out(sh, n_out);
  for (int i = tid; i < k; i += kMergeThreads) {
    int64_t id = -1;
    float s = -INFINITY;
    if (i < n_out) {
      const uint2 e = key_to_entry(sh.out[i]);
      id = static_cast<int64_t>(e.y) + id_offset;
      s = __uint_as_float(e.x);
    }
    out_ids[static_cast<size_t>(q) * k + i] = id;
    out_scores[static_cast<size_t>(q) * k + i] = s;
  }
}

// Lower bound on the k-th largest value of each row (22 leading key bits
// exact, the rest rounded down). NaN counts as -inf. Rows shorter than k: -inf.
// Row q of the input is nseg segments of n floats, segment j at
// vals + j * seg_stride + q * stride (nseg = 1: a plain row-major matrix;
// nseg = W: the [W, B, k] stack of every shard's sample values). out[q] is a
// lower bound on the k-th largest value of the row: the 22-bit prefix of the
// order key of the k-th largest, as a float (-inf when the row holds fewer
// than k values). NaN ranks lowest. With out_vals, also writes k values of the
// row that are >= out[q] (any k of them; -inf pads a row of fewer than k).
__global__ void __launch_bounds__(kMergeThreads) row_kth_kernel(const float* __restrict__ vals, int n, int64_t stride,
                                                                int nseg, int64_t seg_stride, int k,
                                                                float* __restrict__ out,
                                                                float* __restrict__ out_vals) {
  __shared__ SelectShared sh;
  const int q = blockIdx.x;
  const int total = n * nseg;
  auto value_at = [&](int i) -> float {
    const int seg = i / n;
    return vals[seg * seg_stride + static_cast<int64_t>(q) * stride + (i - seg * n)];
  };
  uint32_t prefix = 0, mask = 0;
  if (total >= k) {
    uint32_t need = static_cast<uint32_t>(k);
    for (int shift = 21; shift >= 10; shift -= 11) {
      for (int i = threadIdx.x; i < kBins; i += kMergeThreads) sh.hist[i] = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < total; i += kMergeThreads) {
        const float v = value_at(i);
        const uint32_t key = isnan(v) ? 0u : f2ord(v);
        if ((key & mask) == prefix) atomicAdd(&sh.hist[(key >> shift) & 0x7ffu], 1u);
      }
      __syncthreads();
      block_find_digit_n<kBins / kMergeThreads>(sh, need);
      prefix |= sh.digit << shift;
      mask |= 0x7ffu << shift;
      need -= sh.above;
      __syncthreads();
    }
  }
  const float bound = (prefix <= f2ord_bits(0xff800000u)) ? -INFINITY : ord2f(prefix);
  if (threadIdx.x == 0) {
    out[q] = bound;
    sh.n_out = 0;
  }
  if (out_vals == nullptr) return;
  __syncthreads();
  float* dst = out_vals + static_cast<int64_t>(q) * k;
  for (int i = threadIdx.x; i < total; i += kMergeThreads) {
    const float v = value_at(i);
    const uint32_t key = isnan(v) ? 0u : f2ord(v);
    if (key >= prefix) {
      const uint32_t slot = atomicAdd(&sh.n_out, 1u);
      if (slot < static_cast<uint32_t>(k)) dst[slot] = v;
    }
  }
  __syncthreads();
  for (int i = static_cast<int>(sh.n_out) + threadIdx.x; i < k; i += kMergeThreads) dst[i] = -INFINITY;
}

int row_kth_lower_bound(const float* vals, int B, int n, int64_t stride, int nseg, int64_t seg_stride, int k,
                        float* out, float* out_vals, cudaStream_t stream) {
  if (B == 0) return RB_OK;
  row_kth_kernel<<<B, kMergeThreads, 0, stream>>>(vals, n, stride, nseg, seg_stride, k, out, out_vals);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
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
  (void)out_kth;
  if (k < 1 || k > kMaxK) {
    set_last_error("merge: k must be in [1, 1024]");
    return RB_ERR_INVALID_ARG;
  }
  if (B == 0) return RB_OK;
  merge_lists_kernel<<<B, kMergeThreads, 0, stream>>>(lists, counts, n_lists, stride, k, id_offset, out_ids,
                                                      out_scores);
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
