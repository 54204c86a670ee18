// 1-bit codes -> +-1 int8 rows, so that 1-bit match scores run on the int8
// tensor cores: for q, x in {-1, +1}^(64 W), q . x = 64 W - 2 popcount(q ^ x),
// exactly the score of retrieve::oporp_1bit_match_topk
// (retrieve/src/retrieve/ops/reference/oporp_1bit_match_topk.py:9-41), with the
// bit order of the reference's packers (bit b of word w = coordinate 64 w + b,
// retrieve/src/retrieve/indexing/quantize.py:63-72).
#include <algorithm>
#include <cstdint>

#include "rb_capi_internal.h"

namespace rb {

// Four bits (b0 lowest) -> four bytes, each +1 (0x01) for a set bit and -1
// (0xff) for a clear one, byte j from bit j.
__device__ __forceinline__ uint32_t nibble_pm1(uint32_t nib) {
  // spread bit j to bit 8 j (byte j = 0 or 1), then 0xff ^ (0xfe * byte): 1 ->
  // 0x01, 0 -> 0xff; each byte's product stays inside its byte (no carries)
  const uint32_t spread = (nib & 1u) | ((nib & 2u) << 7) | ((nib & 4u) << 14) | ((nib & 8u) << 21);
  return 0xffffffffu ^ (spread * 0xfeu);
}

// The same in fp8 e4m3: +1.0 is 0x38, -1.0 is 0xb8 (the sign bit set).
__device__ __forceinline__ uint32_t nibble_pm1_e4m3(uint32_t nib) {
  const uint32_t spread = (nib & 1u) | ((nib & 2u) << 7) | ((nib & 4u) << 14) | ((nib & 8u) << 21);
  return 0xb8b8b8b8u ^ (spread * 0x80u);
}

// One thread per 64-bit word: 64 output bytes as four 16-byte stores.
template <bool E4M3>
__global__ void bits_to_pm1_kernel(const uint64_t* __restrict__ bits, int64_t n_words, int4* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_words;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint64_t w = bits[i];
#pragma unroll
    for (int part = 0; part < 4; ++part) {
      const uint32_t v = static_cast<uint32_t>(w >> (16 * part));  // bits 16 part .. 16 part + 15
      int4 o;
      auto nib = [](uint32_t x) { return E4M3 ? nibble_pm1_e4m3(x) : nibble_pm1(x); };
      o.x = static_cast<int>(nib(v & 0xfu));
      o.y = static_cast<int>(nib((v >> 4) & 0xfu));
      o.z = static_cast<int>(nib((v >> 8) & 0xfu));
      o.w = static_cast<int>(nib((v >> 12) & 0xfu));
      out[i * 4 + part] = o;
    }
  }
}

// Sign packing, the last step of the reference's 1-bit projections
// (retrieve/src/retrieve/indexing/quantize.py:63-72 `_pack_signs_to_int64`): bit b
// of word w is set iff values[64 w + b] > 0 (NaN and -0.0 give 0). One warp per
// word: two coalesced 128-byte loads and two ballots, lane 0 stores the word.
__global__ void pack_signs_kernel(const float* __restrict__ values, int64_t n_words, uint64_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); w < n_words; w += warps) {
    const float* v = values + w * 64;
    const uint32_t lo = __ballot_sync(0xffffffffu, v[lane] > 0.f);
    const uint32_t hi = __ballot_sync(0xffffffffu, v[32 + lane] > 0.f);
    if (lane == 0) out[w] = static_cast<uint64_t>(lo) | (static_cast<uint64_t>(hi) << 32);
  }
}

}  // namespace rb

using namespace rb;

static int bits_launch(bool e4m3, const int64_t* bits, int N, int W, void* out, void* stream) {
  if (N < 0 || W <= 0) {
    set_last_error("bits_to_pm1: bad sizes");
    return RB_ERR_INVALID_ARG;
  }
  if (N == 0) return RB_OK;
  if (bits == nullptr || out == nullptr || (reinterpret_cast<uintptr_t>(out) & 15u) != 0) {
    set_last_error("bits_to_pm1: null pointer or output not 16-byte aligned");
    return RB_ERR_INVALID_ARG;
  }
  const int64_t n_words = static_cast<int64_t>(N) * W;
  const int blocks = static_cast<int>(std::min<int64_t>((n_words + 255) / 256, 8 * 1024));
  auto s = static_cast<cudaStream_t>(stream);
  if (e4m3)
    bits_to_pm1_kernel<true><<<blocks, 256, 0, s>>>(reinterpret_cast<const uint64_t*>(bits), n_words,
                                                     reinterpret_cast<int4*>(out));
  else
    bits_to_pm1_kernel<false><<<blocks, 256, 0, s>>>(reinterpret_cast<const uint64_t*>(bits), n_words,
                                                      reinterpret_cast<int4*>(out));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

extern "C" {

int rb_bits_to_pm1(const int64_t* bits, int N, int W, int8_t* out, void* stream) {
  return bits_launch(false, bits, N, W, out, stream);
}

int rb_bits_to_pm1_e4m3(const int64_t* bits, int N, int W, uint8_t* out, void* stream) {
  return bits_launch(true, bits, N, W, out, stream);
}

int rb_pack_signs(const float* values, int64_t M, int D, int64_t* out_words, void* stream) {
  if (M < 0 || D <= 0 || D % 64 != 0) {
    set_last_error("pack_signs: values must be [M, D] with D a positive multiple of 64");
    return RB_ERR_INVALID_ARG;
  }
  const int64_t n_words = M * (D / 64);
  if (n_words == 0) return RB_OK;
  if (values == nullptr || out_words == nullptr) {
    set_last_error("pack_signs: null pointer");
    return RB_ERR_INVALID_ARG;
  }
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((n_words + threads / 32 - 1) / (threads / 32), 148 * 16);
  pack_signs_kernel<<<static_cast<int>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      values, n_words, reinterpret_cast<uint64_t*>(out_words));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

}  // extern "C"
