// SilverTorch's bloom hash and build positions, host and device: MurmurHash3 x64-128 of the
// 16-byte key (feature id, value) with a 64-bit seed, the two halves XOR-ed (Appleby's
// published algorithm, as silvertorch/ops/csrc/bloom_index_util.cuh:61-107 uses it), and the
// first k distinct positions hash % b over seeds 0, 1, ... (bloom_index_util.cuh:185-208).
// bloom.cu builds the indexes with them; tests/native/st_filters_host.cu runs them on the CPU.
#pragma once

#include <cstdint>

#ifdef __CUDACC__
#define RB_HD_HASH __host__ __device__
#else
#define RB_HD_HASH
#endif

namespace rb {

constexpr int kBloomMaxBuildK = 64;    // MAX_K
constexpr int kBloomSeedLimit = 4096;  // seeds tried for k distinct positions

RB_HD_HASH inline uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }

RB_HD_HASH inline uint64_t fmix64(uint64_t k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdull;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ull;
  k ^= k >> 33;
  return k;
}

RB_HD_HASH inline uint64_t murmur3_pair(uint64_t x, uint64_t y, uint64_t seed) {
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

// The first k distinct positions hash(fid, value, seed) % b over seeds 0, 1, ...
// (bloom_index_util.cuh:185-208); at most kBloomSeedLimit seeds are tried.
RB_HD_HASH inline int bloom_build_positions(uint64_t fid, uint64_t value, int64_t b, int k, int64_t* used) {
  int n_used = 0;
  for (int seed = 0; seed < kBloomSeedLimit && n_used < k; ++seed) {
    const int64_t p = static_cast<int64_t>(murmur3_pair(fid, value, static_cast<uint64_t>(seed)) %
                                           static_cast<uint64_t>(b));
    bool dup = false;
    for (int i = 0; i < n_used; ++i) dup |= used[i] == p;
    if (!dup) used[n_used++] = p;
  }
  return n_used;
}

// Bits a doc of a 2048-doc bundle whose docs hold at most max_values values: the configured
// width, or trunc(fp64(max_values * k) * b_multiplier) (bloom_indexer.cpp:60-66,
// bloom_indexer_cuda.cu:330-335).
RB_HD_HASH inline int64_t bloom_bundle_width(int64_t max_values, int k, double b_multiplier, int64_t fixed_b) {
  return fixed_b > 0 ? fixed_b : static_cast<int64_t>(static_cast<double>(max_values * k) * b_multiplier);
}

// Doc d's word for bit row pos of its bundle (bundle rows start at row b0) and its bit:
// bit 63 - d % 64 of word (b0 + pos) * 32 + (d % 2048) / 64.
RB_HD_HASH inline int64_t bloom_word(int64_t b0, int64_t pos, int64_t d) { return (b0 + pos) * 32 + (d % 2048) / 64; }
RB_HD_HASH inline uint64_t bloom_bit(int64_t d) { return 1ull << (63 - (d & 63)); }

}  // namespace rb
