/*
 * C restatements for the oracle (test infrastructure only): sequences whose
 * exact fp32 rounding matters.
 *
 * oracle_gemv: retrieve/src/retrieve/ops/triton/gemv_scores.py:19-28 — per item
 * n, acc = fmaf(q[k], e[k][n], acc) for k = 0 .. D-1, starting at 0.
 */
#include <math.h>
#include <stdint.h>

static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t exp = (h >> 10) & 0x1f;
  const uint32_t man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      int e = -1;
      uint32_t m = man;
      do {
        m <<= 1;
        ++e;
      } while ((m & 0x400) == 0);
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3ff) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  __builtin_memcpy(&f, &bits, 4);
  return f;
}

void oracle_gemv(const uint16_t* q, const uint16_t* et, int64_t D, int64_t N, float* out) {
  for (int64_t n = 0; n < N; ++n) {
    float acc = 0.0f;
    for (int64_t k = 0; k < D; ++k) acc = fmaf(half_to_float(q[k]), half_to_float(et[k * N + n]), acc);
    out[n] = acc;
  }
}
