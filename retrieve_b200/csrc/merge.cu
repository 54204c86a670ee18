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

constexpr int kMaxLists = 1024;

struct SelectShared {
  uint32_t hist[kBins];
  uint32_t warp_tot[kMergeThreads / 32];
  uint32_t digit, above, in_digit;
  uint32_t n_keys, n_out;
  uint64_t kmax, kmin;
  int pre[kMaxLists + 1];  // prefix sums of the list lengths
  uint64_t keys[kSmemKeys];
  uint64_t out[kMaxK];
};

// Finds the digit whose bucket holds the need-th largest element of a
// histogram with nbins = 256 * BPT bins. Thread t owns bins
// [nbins - BPT*(t+1), nbins - BPT*t), so a prefix over threads is a suffix over
// bins. Results land in sh.digit / sh.above / sh.in_digit.
// Shared memory of the row select: the histogram only (8 KB), so that a whole
// B = 1024 batch of rows runs in one wave.
struct RowSelectShared {
  uint32_t hist[kBins];
  uint32_t warp_tot[kMergeThreads / 32];
  uint32_t digit, above, in_digit;
  uint32_t n_out;
};

template <int BPT, class Shared>
__device__ __forceinline__ void block_find_digit_n(Shared& sh, uint32_t need) {
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

// Radix select over 64-bit keys that `visit` enumerates (each thread visits a
// strided share), given that every key agrees with `prefix` on the bits above
// `hi` (prefix's lower bits are zero). 11-bit digits from bit hi down. Returns
// the cut: exactly k keys are >= cut. Requires more than k distinct keys.
template <class Visit>
__device__ uint64_t block_radix_cut(const Visit& visit, int k, int hi, uint64_t prefix, SelectShared& sh) {
  uint64_t mask = (hi >= 63) ? 0ull : ~((2ull << hi) - 1ull);
  uint32_t need = static_cast<uint32_t>(k);
  while (hi >= 0) {
    const int bits = min(11, hi + 1);
    const int shift = hi + 1 - bits;
    const uint64_t dmask = (1ull << bits) - 1ull;
    for (int i = threadIdx.x; i < kBins; i += kMergeThreads) sh.hist[i] = 0;
    __syncthreads();
    visit([&](uint64_t key) {
      if ((key & mask) == prefix) atomicAdd(&sh.hist[(key >> shift) & dmask], 1u);
    });
    __syncthreads();
    block_find_digit_n<kBins / kMergeThreads>(sh, need);
    prefix |= static_cast<uint64_t>(sh.digit) << shift;
    mask |= dmask << shift;
    need -= sh.above;
    const bool done = (sh.in_digit == need);
    __syncthreads();
    if (done) break;
    hi = shift - 1;
  }
  return prefix;
}

// Block max / min of one key per thread (0 / ~0 for threads without one).
__device__ __forceinline__ void block_max_min(uint64_t vmax, uint64_t vmin, SelectShared& sh) {
  for (int off = 16; off > 0; off >>= 1) {
    const uint64_t a = __shfl_xor_sync(RB_FULL_MASK, vmax, off), b = __shfl_xor_sync(RB_FULL_MASK, vmin, off);
    vmax = a > vmax ? a : vmax;
    vmin = b < vmin ? b : vmin;
  }
  if (threadIdx.x == 0) {
    sh.kmax = 0;
    sh.kmin = ~0ull;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    atomicMax(reinterpret_cast<unsigned long long*>(&sh.kmax), static_cast<unsigned long long>(vmax));
    atomicMin(reinterpret_cast<unsigned long long*>(&sh.kmin), static_cast<unsigned long long>(vmin));
  }
  __syncthreads();
}

// Per-query merge of candidate lists into the sorted top-k. List r of query q
// starts at lists + q * q_stride + r * r_stride and holds counts[q * n_lists + r]
// entries (all cap entries when counts is null); an entry is (fp32 score bits,
// uint32 id), id 0xffffffff marks padding. Output: ids + id_offset and scores,
// or (pairs) the same as (score bits, uint32 global id); -1 / -inf (pairs:
// 0xffffffff / -inf) pad rows with fewer than k entries. Score descending, ties
// to the lower id, NaN lowest.
template <bool PAIRS>
__global__ void __launch_bounds__(kMergeThreads) merge_lists_kernel(
    const uint2* __restrict__ lists, const int* __restrict__ counts, int n_lists, int64_t q_stride, int64_t r_stride,
    int cap, int k, int64_t id_offset, int64_t* __restrict__ out_ids, float* __restrict__ out_scores,
    uint2* __restrict__ out_pairs, const int* __restrict__ row_live) {
  __shared__ SelectShared sh;
  const int q = blockIdx.x;
  if (row_live != nullptr && row_live[q] == 0) return;  // the whole block: this row keeps its output
  const int tid = threadIdx.x;
  const uint2* qlists = lists + static_cast<int64_t>(q) * q_stride;

  // list lengths and their prefix sums (warp 0)
  if (tid < 32) {
    int carry = 0;
    for (int r0 = 0; r0 < n_lists; r0 += 32) {
      const int r = r0 + tid;
      int c = 0;
      if (r < n_lists) c = counts ? min(counts[static_cast<int64_t>(q) * n_lists + r], cap) : cap;
      int incl = c;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(RB_FULL_MASK, incl, off);
        if (tid >= off) incl += v;
      }
      if (r < n_lists) sh.pre[r] = carry + incl - c;
      carry += __shfl_sync(RB_FULL_MASK, incl, 31);
    }
    if (tid == 0) {
      sh.pre[n_lists] = carry;
      sh.n_keys = 0;
      sh.n_out = 0;
    }
  }
  __syncthreads();
  const int total = sh.pre[n_lists];
  // every entry, all threads at once: position p lies in list r with
  // pre[r] <= p < pre[r + 1] (binary search over the prefix sums)
  auto visit_global = [&](auto&& f) {
    for (int p = tid; p < total; p += kMergeThreads) {
      int lo = 0, hi = n_lists;
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (sh.pre[mid] <= p) lo = mid; else hi = mid;
      }
      const uint2 v = qlists[lo * r_stride + (p - sh.pre[lo])];
      if (v.y != 0xffffffffu) f(make_key(v.x, v.y));
    }
  };

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

  // 2) exact cut from the highest bit where the keys differ, 3) the <= k
  // winners into sh.out
  if (on_chip) {
    const int n = static_cast<int>(sh.n_keys);
    if (n > k) {
      uint64_t vmax = 0, vmin = ~0ull;
      for (int i = tid; i < n; i += kMergeThreads) {
        const uint64_t key = sh.keys[i];
        vmax = key > vmax ? key : vmax;
        vmin = key < vmin ? key : vmin;
      }
      block_max_min(vmax, vmin, sh);
      const int hi = 63 - __clzll(static_cast<long long>(sh.kmax ^ sh.kmin));
      const uint64_t prefix = (hi >= 63) ? 0ull : (sh.kmax & ~((2ull << hi) - 1ull));
      auto visit_smem = [&](auto&& f) {
        for (int i = tid; i < n; i += kMergeThreads) f(sh.keys[i]);
      };
      const uint64_t cut = block_radix_cut(visit_smem, k, hi, prefix, sh);
      for (int i = tid; i < n; i += kMergeThreads)
        if (sh.keys[i] >= cut) sh.out[atomicAdd(&sh.n_out, 1u)] = sh.keys[i];
    } else {
      for (int i = tid; i < n; i += kMergeThreads) sh.out[i] = sh.keys[i];
      if (tid == 0) sh.n_out = n;
    }
  } else {
    const uint64_t cut = block_radix_cut(visit_global, k, 63, 0ull, sh);
    visit_global([&](uint64_t key) {
      if (key >= cut) sh.out[atomicAdd(&sh.n_out, 1u)] = key;
    });
  }
  __syncthreads();

  // 4) rank sort (keys are distinct): slot = number of larger keys
  const int n_out = min(static_cast<int>(sh.n_out), k);
  for (int i = tid; i < n_out; i += kMergeThreads) {
    const uint64_t key = sh.out[i];
    int rank = 0;
    for (int j = 0; j < n_out; ++j) rank += (sh.out[j] > key);
    sh.keys[rank] = key;
  }
  __syncthreads();
  for (int i = tid; i < k; i += kMergeThreads) {
    const size_t o = static_cast<size_t>(q) * k + i;
    if constexpr (PAIRS) {
      uint2 e = make_uint2(0xff800000u, 0xffffffffu);
      if (i < n_out) {
        e = key_to_entry(sh.keys[i]);
        e.y = static_cast<uint32_t>(static_cast<int64_t>(e.y) + id_offset);
      }
      out_pairs[o] = e;
    } else {
      int64_t id = -1;
      float sc = -INFINITY;
      if (i < n_out) {
        const uint2 e = key_to_entry(sh.keys[i]);
        id = static_cast<int64_t>(e.y) + id_offset;
        sc = __uint_as_float(e.x);
      }
      out_ids[o] = id;
      out_scores[o] = sc;
    }
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
  __shared__ RowSelectShared sh;
  const int q = blockIdx.x;
  const int total = n * nseg;
  // every value of the row once, each thread a strided share of every segment
  auto for_each = [&](auto&& f) {
    for (int seg = 0; seg < nseg; ++seg) {
      const float* row = vals + seg * seg_stride + static_cast<int64_t>(q) * stride;
      for (int i = threadIdx.x; i < n; i += kMergeThreads) f(row[i]);
    }
  };
  uint32_t prefix = 0, mask = 0;
  if (total >= k) {
    uint32_t need = static_cast<uint32_t>(k);
    for (int shift = 21; shift >= 10; shift -= 11) {
      for (int i = threadIdx.x; i < kBins; i += kMergeThreads) sh.hist[i] = 0;
      __syncthreads();
      for_each([&](float v) {
        const uint32_t key = isnan(v) ? 0u : f2ord(v);
        if ((key & mask) == prefix) atomicAdd(&sh.hist[(key >> shift) & 0x7ffu], 1u);
      });
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
  for_each([&](float v) {
    const uint32_t key = isnan(v) ? 0u : f2ord(v);
    if (key >= prefix) {
      const uint32_t slot = atomicAdd(&sh.n_out, 1u);
      if (slot < static_cast<uint32_t>(k)) dst[slot] = v;
    }
  });
  __syncthreads();
  for (int i = static_cast<int>(sh.n_out) + threadIdx.x; i < k; i += kMergeThreads) dst[i] = -INFINITY;
}

// Two lower bounds per row in one read pair: out1[q] / out2[q] bound the k1-th / k2-th largest
// value of row q (-inf where the row holds fewer), with row_kth_kernel's 22-bit precision.
// The top 11 bits' histogram serves both ranks; the next 11 bits get one histogram each.
__global__ void __launch_bounds__(kMergeThreads) row_kth2_kernel(const float* __restrict__ vals, int n, int64_t stride,
                                                                 int k1, int k2, float* __restrict__ out1,
                                                                 float* __restrict__ out2) {
  __shared__ RowSelectShared sh[2];
  const int q = blockIdx.x;
  const float* row = vals + static_cast<int64_t>(q) * stride;
  const int kk[2] = {k1, k2};
  uint32_t prefix[2] = {0u, 0u}, need[2] = {static_cast<uint32_t>(k1), static_cast<uint32_t>(k2)};
  if (n >= min(k1, k2)) {
    for (int i = threadIdx.x; i < kBins; i += kMergeThreads) sh[0].hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kMergeThreads) {
      const float v = row[i];
      atomicAdd(&sh[0].hist[(isnan(v) ? 0u : f2ord(v)) >> 21], 1u);
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (n >= kk[t]) {  // block-uniform
        block_find_digit_n<kBins / kMergeThreads>(sh[0], need[t]);
        prefix[t] = sh[0].digit << 21;
        need[t] -= sh[0].above;
      }
      __syncthreads();
    }
    for (int i = threadIdx.x; i < kBins; i += kMergeThreads) sh[0].hist[i] = sh[1].hist[i] = 0;
    __syncthreads();
    const uint32_t mask = 0x7ffu << 21;
    for (int i = threadIdx.x; i < n; i += kMergeThreads) {
      const float v = row[i];
      const uint32_t key = isnan(v) ? 0u : f2ord(v);
      if (n >= k1 && (key & mask) == prefix[0]) atomicAdd(&sh[0].hist[(key >> 10) & 0x7ffu], 1u);
      if (n >= k2 && (key & mask) == prefix[1]) atomicAdd(&sh[1].hist[(key >> 10) & 0x7ffu], 1u);
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (n >= kk[t]) {
        block_find_digit_n<kBins / kMergeThreads>(sh[t], need[t]);
        prefix[t] |= sh[t].digit << 10;
      }
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) {
    out1[q] = (n < k1 || prefix[0] <= f2ord_bits(0xff800000u)) ? -INFINITY : ord2f(prefix[0]);
    out2[q] = (n < k2 || prefix[1] <= f2ord_bits(0xff800000u)) ? -INFINITY : ord2f(prefix[1]);
  }
}

int row_kth2_lower_bounds(const float* vals, int B, int n, int64_t stride, int k1, int k2, float* out1, float* out2,
                          cudaStream_t stream) {
  if (B == 0) return RB_OK;
  row_kth2_kernel<<<B, kMergeThreads, 0, stream>>>(vals, n, stride, k1, k2, out1, out2);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
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

static int merge_launch(const uint2* lists, const int* counts, int B, int n_lists, int64_t q_stride,
                        int64_t r_stride, int cap, int k, int64_t id_offset, int64_t* out_ids, float* out_scores,
                        uint2* out_pairs, cudaStream_t stream, const int* row_live = nullptr) {
  if (k < 1 || k > kMaxK) {
    set_last_error("merge: k must be in [1, 1024]");
    return RB_ERR_INVALID_ARG;
  }
  if (n_lists < 1 || n_lists > kMaxLists) {
    set_last_error("merge: between 1 and 1024 lists per query");
    return RB_ERR_INVALID_ARG;
  }
  if (B == 0) return RB_OK;
  if (out_pairs != nullptr)
    merge_lists_kernel<true><<<B, kMergeThreads, 0, stream>>>(lists, counts, n_lists, q_stride, r_stride, cap, k,
                                                               id_offset, nullptr, nullptr, out_pairs, row_live);
  else
    merge_lists_kernel<false><<<B, kMergeThreads, 0, stream>>>(lists, counts, n_lists, q_stride, r_stride, cap, k,
                                                                id_offset, out_ids, out_scores, nullptr, row_live);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int merge_lists(const uint2* lists, const int* counts, int B, int n_lists, int stride, int k, int64_t id_offset,
                int64_t* out_ids, float* out_scores, uint2* out_pairs, cudaStream_t stream, const int* row_live) {
  return merge_launch(lists, counts, B, n_lists, static_cast<int64_t>(n_lists) * stride, stride, stride, k, id_offset,
                      out_ids, out_scores, out_pairs, stream, row_live);
}

int merge_pair_stack(const uint2* pairs, int W, int B, int kin, int k, int64_t* out_ids, float* out_scores,
                     cudaStream_t stream) {
  return merge_launch(pairs, nullptr, B, W, kin, static_cast<int64_t>(B) * kin, kin, k, 0, out_ids, out_scores,
                      nullptr, stream);
}

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

__global__ void fill_empty_pairs_kernel(uint2* out, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = make_uint2(0xff800000u, 0xffffffffu);
}

void fill_empty_pairs(uint2* out, size_t n, cudaStream_t stream) {
  if (n == 0) return;
  const int blocks = static_cast<int>(std::min<size_t>((n + 255) / 256, 1024));
  fill_empty_pairs_kernel<<<blocks, 256, 0, stream>>>(out, n);
}

void fill_empty(int64_t* out_ids, float* out_scores, size_t n, cudaStream_t stream) {
  if (n == 0) return;
  const int blocks = static_cast<int>(std::min<size_t>((n + 255) / 256, 1024));
  fill_empty_kernel<<<blocks, 256, 0, stream>>>(out_ids, out_scores, n);
}

}  // namespace rb
