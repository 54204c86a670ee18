// Per-item 64-bit Bloom words, built on the device (index build time).
// Hash: MurmurHash3 x64-128 of the 16-byte key (clause, value) with a 64-bit
// seed, halves XOR-ed (Appleby's published algorithm, as silvertorch
// bloom_index_util.cuh:61-107 uses it); positions: the first k distinct
// hash % 64 for seed = 0, 1, ... (bloom_index_util.cuh:185-208).
#include <algorithm>
#include <cstdint>

#include "bloom_hash.cuh"
#include "rb_capi_internal.h"

namespace rb {

__global__ void bloom_build_kernel(const int64_t* __restrict__ attrs, int N, int C, int A, int k,
                                   uint64_t* __restrict__ words) {
  for (int64_t n = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; n < N;
       n += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint64_t w = 0;
    const int64_t* row = attrs + n * C * A;
    for (int c = 0; c < C; ++c) {
      for (int a = 0; a < A; ++a) {
        const int64_t v = row[c * A + a];
        if (v == -1) continue;
        uint64_t used = 0;
        int got = 0;
        for (uint64_t seed = 0; got < k && seed < 4096; ++seed) {
          const uint64_t bit = 1ull << (murmur3_pair(static_cast<uint64_t>(c), static_cast<uint64_t>(v), seed) % 64);
          if (!(used & bit)) {
            used |= bit;
            ++got;
          }
        }
        w |= used;
      }
    }
    words[n] = w;
  }
}

// The per-item words bit-sliced for the filtered dense scan: per 32-item chunk c,
// word p (of 64) holds bit p of items 32 c .. 32 c + 31 (bit j = item 32 c + j);
// chunks past N (up to whole 128-item tiles) are zero. One warp per chunk: 64
// ballots, then lane l stores words l and l + 32.
__global__ void bloom_slices_kernel(const uint64_t* __restrict__ words, int64_t N, int64_t n_chunks,
                                    uint32_t* __restrict__ slices) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); c < n_chunks;
       c += warps) {
    const int64_t item = 32 * c + lane;
    const uint64_t w = item < N ? words[item] : 0ull;
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int pos = 0; pos < 32; ++pos) {
      const uint32_t b0 = __ballot_sync(0xffffffffu, (w >> pos) & 1ull);
      const uint32_t b1 = __ballot_sync(0xffffffffu, (w >> (pos + 32)) & 1ull);
      if (lane == pos) {
        lo = b0;
        hi = b1;
      }
    }
    slices[64 * c + lane] = lo;
    slices[64 * c + 32 + lane] = hi;
  }
}

size_t bloom_slices_bytes(int64_t N) {
  const int64_t tiles = (N + 127) / 128;
  return static_cast<size_t>(tiles) * 4 * 64 * sizeof(uint32_t);
}

int bloom_slices(const uint64_t* words, int64_t N, uint32_t* slices, cudaStream_t stream) {
  const int64_t n_chunks = (N + 127) / 128 * 4;
  if (n_chunks == 0) return RB_OK;
  const int64_t blocks = std::min<int64_t>((n_chunks + 7) / 8, 4096);
  bloom_slices_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(words, N, n_chunks, slices);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// SilverTorch's bundle-major bloom index (st::bloom_index_build and the CUDA-only
// st::bloom_index_build_fixed; silvertorch/ops/csrc/bloom_indexer.cpp:26-114,
// bloom_indexer_cuda.cu:291-340, 790-960). Input: the jagged feature layout
// (feature_ids int32 [C]; feature_offsets int64 [N C + 1], CSR over (doc, feature);
// feature_values int64). Docs fall in bundles of 2048; bundle i is
// B_i = fixed_b, or trunc(fp64(max values of a doc in the bundle * k) * b_multiplier)
// bits per doc; bundle_b_offsets is the prefix sum of the B_i. Each value of feature f
// sets, for its first k distinct positions p = hash(f, value, seed) % B_i over seeds
// 0, 1, ..., bit 63 - d % 64 of word (bundle_b_offsets[i] + p) * 32 + (d % 2048) / 64.
// ---------------------------------------------------------------------------
constexpr int kBundleDocs = 2048;
constexpr int kBloomThreads = 256;

__global__ void __launch_bounds__(kBloomThreads) bloom_bundle_width_kernel(
    const int64_t* __restrict__ feature_offsets, int64_t N, int C, int k, double b_multiplier, int64_t fixed_b,
    int64_t* __restrict__ widths) {
  __shared__ int64_t red[kBloomThreads / 32];
  const int64_t bundle = blockIdx.x;
  int64_t m = 0;
  for (int64_t d = bundle * kBundleDocs + threadIdx.x; d < min(N, (bundle + 1) * kBundleDocs); d += kBloomThreads) {
    const int64_t cnt = feature_offsets[(d + 1) * C] - feature_offsets[d * C];
    m = max(m, cnt);
  }
  for (int off = 16; off > 0; off >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t mm = 0;
    for (int w = 0; w < kBloomThreads / 32; ++w) mm = max(mm, red[w]);
    widths[bundle] = bloom_bundle_width(mm, k, b_multiplier, fixed_b);
  }
}

// bundle_b_offsets[0] = 0, bundle_b_offsets[i + 1] = bundle_b_offsets[i] + widths[i]; one CTA.
__global__ void __launch_bounds__(kBloomThreads) bloom_bundle_scan_kernel(const int64_t* __restrict__ widths,
                                                                          int64_t n, int64_t* __restrict__ offsets) {
  __shared__ int64_t part[kBloomThreads];
  const int tid = threadIdx.x;
  const int64_t per = (n + kBloomThreads - 1) / kBloomThreads;
  const int64_t i0 = min(n, tid * per), i1 = min(n, i0 + per);
  int64_t sum = 0;
  for (int64_t i = i0; i < i1; ++i) sum += widths[i];
  part[tid] = sum;
  __syncthreads();
  for (int off = 1; off < kBloomThreads; off <<= 1) {
    const int64_t v = tid >= off ? part[tid - off] : 0;
    __syncthreads();
    part[tid] += v;
    __syncthreads();
  }
  int64_t run = part[tid] - sum;
  if (tid == 0) offsets[0] = 0;
  for (int64_t i = i0; i < i1; ++i) {
    run += widths[i];
    offsets[i + 1] = run;
  }
}

// One thread per doc: every value of every feature sets its k positions.
__global__ void bloom_index_fill_kernel(const int32_t* __restrict__ feature_ids,
                                        const int64_t* __restrict__ feature_offsets,
                                        const int64_t* __restrict__ feature_values, int64_t n_values, int64_t N,
                                        int C, int k, const int64_t* __restrict__ bundle_offsets,
                                        unsigned long long* __restrict__ index, int64_t index_words) {
  for (int64_t d = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; d < N;
       d += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t bundle = d / kBundleDocs;
    const int64_t b0 = bundle_offsets[bundle];
    const int64_t bb = bundle_offsets[bundle + 1] - b0;
    if (bb <= 0) continue;
    const unsigned long long bit = bloom_bit(d);
    for (int c = 0; c < C; ++c) {
      const uint64_t fid = static_cast<uint64_t>(static_cast<int64_t>(feature_ids[c]));
      const int64_t v0 = max(feature_offsets[d * C + c], int64_t{0});
      const int64_t v1 = min(feature_offsets[d * C + c + 1], n_values);
      for (int64_t v = v0; v < v1; ++v) {
        const uint64_t value = static_cast<uint64_t>(feature_values[v]);
        int64_t used[kBloomMaxBuildK];
        const int n_used = bloom_build_positions(fid, value, bb, k, used);
        for (int i = 0; i < n_used; ++i) {
          const int64_t w = bloom_word(b0, used[i], d);
          if (w >= 0 && w < index_words) atomicOr(index + w, bit);
        }
      }
    }
  }
}

}  // namespace rb

using namespace rb;

extern "C" int rb_bloom_slices_bytes(int64_t N, size_t* bytes) {
  if (bytes == nullptr || N < 0) {
    rb::set_last_error("bloom_slices_bytes: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  *bytes = rb::bloom_slices_bytes(N);
  return RB_OK;
}

extern "C" int rb_bloom_slices(const uint64_t* item_bloom, int64_t N, uint32_t* out_slices, void* stream) {
  if (N < 0 || (N > 0 && (item_bloom == nullptr || out_slices == nullptr))) {
    rb::set_last_error("bloom_slices: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  if ((reinterpret_cast<uintptr_t>(out_slices) & 15u) != 0) {
    rb::set_last_error("bloom_slices: out_slices must be 16-byte aligned");
    return RB_ERR_INVALID_ARG;
  }
  if (rb::bloom_slices(item_bloom, N, out_slices, static_cast<cudaStream_t>(stream)) != RB_OK) {
    rb::set_last_error("bloom_slices: launch failed");
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

extern "C" int rb_bloom_build(const int64_t* item_attrs, int N, int C, int A, int k, uint64_t* out_words,
                              void* stream) {
  if (N < 0 || C <= 0 || A <= 0 || k < 1 || k > 64) {
    set_last_error("bloom_build: bad sizes or k");
    return RB_ERR_INVALID_ARG;
  }
  if (N == 0) return RB_OK;
  const int blocks = std::min((N + 255) / 256, 8 * num_sms());
  bloom_build_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(item_attrs, N, C, A, k, out_words);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

extern "C" int rb_bloom_index_widths(const int64_t* feature_offsets, int64_t N, int C, int k, double b_multiplier,
                                     int64_t bits_per_doc, int64_t* widths, int64_t* bundle_b_offsets,
                                     void* stream) {
  if (N < 0 || C <= 0 || k < 1 || k > kBloomMaxBuildK || (bits_per_doc <= 0 && !(b_multiplier > 1.0))) {
    set_last_error("bloom_index_build: bad sizes (k in [1, 64], b_multiplier > 1 or bits_per_doc > 0)");
    return RB_ERR_INVALID_ARG;
  }
  if (bits_per_doc > 0 && bits_per_doc < k) {
    set_last_error("bloom_index_build: bits_per_doc must be at least k");
    return RB_ERR_INVALID_ARG;
  }
  const int64_t n_bundles = (N + kBundleDocs - 1) / kBundleDocs;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_bundles > 0)
    bloom_bundle_width_kernel<<<static_cast<unsigned>(n_bundles), kBloomThreads, 0, s>>>(
        feature_offsets, N, C, k, b_multiplier, bits_per_doc, widths);
  bloom_bundle_scan_kernel<<<1, kBloomThreads, 0, s>>>(widths, n_bundles, bundle_b_offsets);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

extern "C" int rb_bloom_index_fill(const int32_t* feature_ids, const int64_t* feature_offsets,
                                   const int64_t* feature_values, int64_t n_values, int64_t N, int C, int k,
                                   const int64_t* bundle_b_offsets, int64_t* bloom_index, int64_t index_words,
                                   void* stream) {
  if (N < 0 || C <= 0 || k < 1 || k > kBloomMaxBuildK || n_values < 0 || index_words < 0) {
    set_last_error("bloom_index_build: bad sizes");
    return RB_ERR_INVALID_ARG;
  }
  if (N == 0) return RB_OK;
  const int blocks = static_cast<int>(std::min<int64_t>((N + 255) / 256, 148 * 16));
  bloom_index_fill_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      feature_ids, feature_offsets, feature_values, n_values, N, C, k, bundle_b_offsets,
      reinterpret_cast<unsigned long long*>(bloom_index), index_words);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}
