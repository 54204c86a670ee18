// Per-item 64-bit Bloom words, built on the device (index build time).
// Hash: MurmurHash3 x64-128 of the 16-byte key (clause, value) with a 64-bit
// seed, halves XOR-ed (Appleby's published algorithm, as silvertorch
// bloom_index_util.cuh:61-107 uses it); positions: the first k distinct
// hash % 64 for seed = 0, 1, ... (bloom_index_util.cuh:185-208).
#include <algorithm>
#include <cstdint>

#include "rb_capi_internal.h"

namespace rb {

__device__ __forceinline__ uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }

__device__ __forceinline__ uint64_t fmix64(uint64_t k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return k;
}

__device__ __forceinline__ uint64_t murmur3_pair(uint64_t x, uint64_t y, uint64_t seed) {
  const uint64_t c1 = 0x87c37b91114253d5ull, c2 = 0x4cf5ad432745937full;
  uint64_t h1 = seed, h2 = seed;
  uint64_t k1 = rotl64(x * c1, 31) * c2;
  h1 ^= k1;
  h1 = rotl64(h1, 27) + h2;
  h1 = h1 * 5 + 0x52dce729ull;
  uint64_t k2 = rotl64(y * c2, 33) * c1;
  h2 ^= k2;
  h2 = rotl64(h2, 31) + h1;
  h2 = h2 * 5 + 0x38495ab5ull;
  h1 ^= 16;
  h2 ^= 16;
  h1 += h2;
  h2 += h1;
  h1 = fmix64(h1);
  h2 = fmix64(h2);
  h1 += h2;
  h2 += h1;
  return h1 ^ h2;
}

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

}  // namespace rb

using namespace rb;

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
