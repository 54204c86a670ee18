// Fused dense scoring + exact top-k for sm_100a (B200): the kernels. Each
// element type's variants are instantiated in their own translation unit
// (dense_scan_e<ELEM>.cu); the planning and dispatch live in dense_scan_sm100.cu.
//
// Element types (ELEM): 0 fp16, 1 bf16, 2 int8 (kind::i8, int32 accumulate,
// (dot * q_scale) * item_scale dequant), 4 fp8 e4m3 (kind::f8f6f4, unscaled;
// +-1 codes give exact 1-bit match scores). The fp16 and fp8 descriptors share
// their format code 0 (F16 for kind::f16, E4M3 for kind::f8f6f4).
//
// One persistent CTA per SM. A task is (query group, item split): the CTA
// holds NG x 128 queries resident in shared memory (TMA, 128-byte swizzle) and
// streams its split's item tiles (128 items each) through a STAGES-deep TMA
// ring. One elected thread issues tcgen05.mma (M = 128 queries, N = 128 items,
// K = the embedding dim) into a double-buffered TMEM accumulator; the epilogue
// warps read their query row out of TMEM (thread = query, 32 columns at a
// time), drop every 32-item chunk whose max is below the query's threshold and
// append the rest to the query's candidate list (rb_select.cuh). No [B, N]
// score matrix ever reaches HBM.
//
// Warp roles (NG = 2: 320 threads):
//   warp 0      TMA producer (queries once per task, item tiles per stage)
//   warp 1      TMEM allocator + MMA issuer
//   warps 2..   epilogue, 4 warps per query group (TMEM lane quadrant = warp % 4)
//
// Reference semantics replaced: PostfilterKNN.score + masked_topk
// (retrieve/src/retrieve/modules/knn.py:62-76, functional.py:57-85), i.e.
// torch.mm(q_fp16, E_t, out_dtype=fp32) followed by torch.topk, with ties broken
// toward the lower item id.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "rb_capi_internal.h"
#include "rb_common.cuh"
#include "rb_select.cuh"

namespace rb {

constexpr int kTileItems = 128;  // N of one MMA = items per pipeline stage
constexpr int kQTile = 128;      // M of one MMA = queries per group
constexpr int kSampleStride = 16;  // sampling pass: every 16th tile
constexpr int kMaxSmemPerCta = 232448;  // opt-in dynamic shared memory of one CTA on sm_100 (227 KB)

struct alignas(64) DenseScanParams {
  CUtensorMap tmap_q;
  CUtensorMap tmap_x;   // item boxes of 128 rows (1-SM kernel) or 64 rows (2-SM kernel)
  const float* seed;  // [B] pass threshold per query (>=), or null for -inf
  uint2* lists;       // [B, n_splits, cap]
  int* counts;        // [B, n_splits]
  int* err;           // device error word
  float* chunk_max;   // MODE 1: [B, chunk_stride] max score of every 32-item chunk
  int chunk_stride;
  const float* q_scale;  // scaled types: [B] per-query scale (null: 1)
  const float* x_scale;  // scaled types: [N] per-item scale (null: 1)
  FilterArgs filter;     // attribute predicate (mode kFilterNone: none)
  int B, N;
  int n_qsg, n_splits;
  int tile_stride, tile_offset, pass_tiles;
  int k, cap;
  const int* qsg_live;  // null: every query group; else only groups with a nonzero entry are scanned
  int ring;             // 2-SM filtered kernel: bit 0 the Bloom slices, bit 1 the attribute rows of
                        // each tile come through the shared-memory ring (host: dense_scan_pass)
};

__device__ __forceinline__ bool task_live(const DenseScanParams& p, int t) {
  return p.qsg_live == nullptr || p.qsg_live[t % p.n_qsg] != 0;
}

// Bit-sliced Bloom words of one 128-item tile: 4 chunks x 64 words.
constexpr int kTileSliceWords = 4 * 64;

// The 2-SM filtered kernel's ring: kRingSlots tiles in flight, each its 1 KB of Bloom slices
// and up to 8 KB of attribute rows (128 items of at most 8 int64 cells).
constexpr int kRingSlots = 4;
constexpr int kRingRowBytes = kTileItems * 8 * 8;
constexpr int kRingSlotBytes = kTileSliceWords * 4 + kRingRowBytes;

// A filtered chunk whose threshold test passes in at most this many lanes is appended by the
// whole warp (warp_filter_append); with more, each lane tests its own items. Measured at 10M
// items (C3, queries/s at 1 / 10 / 50 % selectivity): 74.5k / 188k / 254k with 4, 83.4k /
// 190k / 253k with 1, 87.3k / 195k / 239k with 0 (per-lane only).
constexpr int kCoopFilterLanes = 1;

// One tile's bit-sliced Bloom words into this warp's buffer (pt & 1) of two, 32 bytes a
// lane (cp.async, committed by the caller).
__device__ __forceinline__ void copy_tile_slices(uint32_t* sl_base, const DenseScanParams& p, int pt, int lane) {
  const size_t tile = static_cast<size_t>(pt * p.tile_stride + p.tile_offset);
  const uint32_t* src = p.filter.slices + tile * kTileSliceWords + lane * 8;
  uint32_t* dst = sl_base + (pt & 1) * kTileSliceWords + lane * 8;
  cp_async16(dst, src);
  cp_async16(dst + 4, src + 4);
}

template <int KB, int NG, int STAGES, bool FILT = false>
struct DenseSmemLayout {
  static constexpr int kOpTile = kQTile * 128;  // bytes of one 128-row x 128-byte K-block
  static constexpr int kA = NG * KB * kOpTile;
  static constexpr int kB = STAGES * KB * kOpTile;
  static constexpr int kEpiWarps = 4 * NG;
  static constexpr int kHist = kEpiWarps * 256 * 4;
  static constexpr int kSlices = FILT ? kEpiWarps * 2 * kTileSliceWords * 4 : 0;  // two tiles' slices a warp
  static constexpr int kBar = (2 * STAGES + 2 + 4 + 1) * 8;
  static constexpr int kMisc = 16;
  static constexpr int kTotal = kA + kB + kHist + kSlices + kBar + kMisc + 1024;  // + alignment slack
};

__device__ __forceinline__ void split_range(int split, int n_splits, int pass_tiles, int& lo, int& hi) {
  lo = static_cast<int>((static_cast<int64_t>(split) * pass_tiles) / n_splits);
  hi = static_cast<int>((static_cast<int64_t>(split + 1) * pass_tiles) / n_splits);
}

// Filtering work of one accumulator tile, on the scores already in registers
// (r[ch][j] = score of item row0 + 32*ch + j for this thread's query).
// Filtering work on NCH 32-item chunks of scores already in registers:
// r[ch][j] = score of item row0 + 32 * ch + j for this thread's query; the
// chunks are chunk numbers c0 .. c0 + NCH - 1 of their 128-item tile.
// The scaled element types dequantize first: score = (fp32(dot) * q_scale) *
// item_scale, left to right as the reference does (ops/official/adapter.py:
// 338-367). For int8 (ELEM 2) the registers hold int32 dots, turned here into
// fp32 exactly; for integer values held as bf16 (ELEM 3) or fp8 e4m3 (ELEM 4)
// the fp32 accumulator already holds the exact integer dot (every partial sum
// is an integer below 2^24).
// int8 (ELEM 2) scores (fp32(dot) * q_scale) * item_scale, left to right as the
// reference dequantizes (ops/official/adapter.py:338-367); null scale arrays
// mean 1. The registers hold int32 dots, turned into fp32 exactly. fp8 e4m3
// (ELEM 4) is unscaled: the fp32 accumulator is the score.
template <int ELEM, int KB>
__device__ __forceinline__ float raw_to_float(uint32_t raw) {
  if constexpr (ELEM != 2)
    return __uint_as_float(raw);
  else if constexpr (KB <= 2)
    return __uint_as_float(raw + 0x4B400000u) - 12582912.0f;  // |dot| < 2^22: exact magic-constant path
  else
    return __int2float_rn(static_cast<int>(raw));  // D = 512: |dot| < 2^24, exact by conversion
}

// `stage` is the calling warp's 1 KB of shared scratch (its list-compaction
// histogram, idle here): the int8 path stages the tile's 128 item scales in it.
// The filtered variants (FILT) with `use_sl` test the Bloom form of the query's
// predicate (`st`) on the tile's bit-sliced Bloom words `sl` (shared memory, 64
// words a chunk), a chunk of 32 items per term and AND; the exact form (recheck
// mode), and queries without `use_sl`, test item by item from global memory.
// The filtered sampling pass with an exact recheck: the best Bloom-passing item of the tile
// seen so far (score NaN: none yet).
struct TileBest {
  float sc;
  uint32_t id;
};

// int8: this lane's four item scales of a tile (items row0 + 4 lane .. + 3; 0 past N) and
// the query's scale, loaded one tile ahead by the epilogue loop so that the loads' latency
// hides behind the previous tile's work.
struct ScalePrefetch {
  float4 xs;
  float qs;
  bool on;
};

__device__ __forceinline__ float4 load_tile_scales(const DenseScanParams& p, uint32_t row0) {
  const uint32_t id = row0 + 4u * (threadIdx.x & 31);
  if (p.x_scale == nullptr) return make_float4(1.f, 1.f, 1.f, 1.f);
  if (row0 + kTileItems <= static_cast<uint32_t>(p.N)) return __ldg(reinterpret_cast<const float4*>(p.x_scale + id));
  float4 v;
  v.x = id < static_cast<uint32_t>(p.N) ? p.x_scale[id] : 0.f;
  v.y = id + 1 < static_cast<uint32_t>(p.N) ? p.x_scale[id + 1] : 0.f;
  v.z = id + 2 < static_cast<uint32_t>(p.N) ? p.x_scale[id + 2] : 0.f;
  v.w = id + 3 < static_cast<uint32_t>(p.N) ? p.x_scale[id + 3] : 0.f;
  return v;
}

template <int MODE, int NCH, int ELEM, bool FILT, int KB>
__device__ __forceinline__ void process_chunks(const DenseScanParams& p, uint32_t (&r)[NCH][32], uint32_t row0,
                                               int chunk0, bool valid_q, int q, float thresh, int& count,
                                               uint2* list, uint32_t* stage, const uint32_t* sl,
                                               const SlicedTerms& st, bool use_sl, TileBest& tb,
                                               const int64_t* tile_rows = nullptr,
                                               const ExactTerm* wterms = nullptr, int ent = 0,
                                               ScalePrefetch sp = ScalePrefetch{}) {
  // Chunks whose scores may pass (bit ch); the full int8 pass clears the bits of
  // chunks it proves below the threshold before dequantizing them.
  uint32_t live = (1u << NCH) - 1u;
  if constexpr (ELEM == 2) {
    const float qs = sp.on ? sp.qs : (!valid_q ? 0.f : (p.q_scale != nullptr ? p.q_scale[q] : 1.f));
    const bool unit_x = p.x_scale == nullptr;
    // Every lane needs all 128 item scales of the tile: the warp loads them
    // once (one float4 per lane, coalesced) into shared memory, and each lane
    // then reads them as broadcasts instead of 32 dependent global loads.
    float4* sx = reinterpret_cast<float4*>(stage);
    float lmax = 1.f, lmin = 1.f;  // this lane's 4 scales' max and min (chunk lane / 8)
    if (!unit_x) {
      const int lane = threadIdx.x & 31;
      float4 v;
      if (sp.on) {
        v = sp.xs;
      } else {
        const uint32_t id = row0 + 4 * static_cast<uint32_t>(lane);
        if (row0 + NCH * 32 <= static_cast<uint32_t>(p.N)) {
          v = __ldg(reinterpret_cast<const float4*>(p.x_scale + id));
        } else {
          v.x = id < static_cast<uint32_t>(p.N) ? p.x_scale[id] : 0.f;
          v.y = id + 1 < static_cast<uint32_t>(p.N) ? p.x_scale[id + 1] : 0.f;
          v.z = id + 2 < static_cast<uint32_t>(p.N) ? p.x_scale[id + 2] : 0.f;
          v.w = id + 3 < static_cast<uint32_t>(p.N) ? p.x_scale[id + 3] : 0.f;
        }
      }
      sx[lane] = v;
      lmax = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
      lmin = fminf(fminf(v.x, v.y), fminf(v.z, v.w));
    }
    if constexpr (MODE == 0 && NCH == 4) {
      // A bound per chunk before any dequantization. With q_scale >= 0 and the
      // chunk's item scales in [xmin, xmax], xmin >= 0, every rounded product is
      // monotonic, so each score fl(fl(dot * qs) * x) is at most fl(A * xmax)
      // (A >= 0) or fl(A * xmin) (A < 0), A = fl(fl(max dot) * qs). A chunk whose
      // bound is below the threshold for every lane is never dequantized. NaN
      // scales or scales below zero leave the chunk live.
#pragma unroll
      for (int off = 4; off >= 1; off >>= 1) {
        lmax = fmaxf(lmax, __shfl_xor_sync(RB_FULL_MASK, lmax, off));
        lmin = fminf(lmin, __shfl_xor_sync(RB_FULL_MASK, lmin, off));
      }
      uint32_t need = 0;
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        const float xmax = __shfl_sync(RB_FULL_MASK, lmax, 8 * ch), xmin = __shfl_sync(RB_FULL_MASK, lmin, 8 * ch);
        int m[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) m[i] = max(static_cast<int>(r[ch][2 * i]), static_cast<int>(r[ch][2 * i + 1]));
#pragma unroll
        for (int w = 8; w >= 1; w >>= 1) {
#pragma unroll
          for (int i = 0; i < w; ++i) m[i] = max(m[2 * i], m[2 * i + 1]);
        }
        const float a = __fmul_rn(raw_to_float<ELEM, KB>(static_cast<uint32_t>(m[0])), qs);
        const bool monotone = qs >= 0.f && xmin >= 0.f;
        const float bound = a >= 0.f ? __fmul_rn(a, xmax) : __fmul_rn(a, xmin);
        if (valid_q && (!monotone || !(bound < thresh))) need |= 1u << ch;
      }
      // the warp dequantizes a chunk if any lane may pass in it (the scales are shared)
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch)
        if (!__any_sync(RB_FULL_MASK, (need >> ch) & 1u)) live &= ~(1u << ch);
    }
    __syncwarp();
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      if (!((live >> ch) & 1u)) continue;  // warp-uniform
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 xs = unit_x ? make_float4(1.f, 1.f, 1.f, 1.f) : sx[ch * 8 + j4];
        const float xv[4] = {xs.x, xs.y, xs.z, xs.w};
#pragma unroll
        for (int u = 0; u < 4; ++u)
          r[ch][4 * j4 + u] =
              __float_as_uint(__fmul_rn(__fmul_rn(raw_to_float<ELEM, KB>(r[ch][4 * j4 + u]), qs), xv[u]));
      }
    }
    __syncwarp();  // every lane has read the staged scales before the scratch is reused
  }
  if (row0 + NCH * 32 > static_cast<uint32_t>(p.N)) {
    // last, partial tile: rows past N were zero-filled by TMA; NaN never passes
    // a threshold test and is ignored by fmaxf
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (row0 + ch * 32 + j >= static_cast<uint32_t>(p.N)) r[ch][j] = 0x7fc00000u;
  }
  if constexpr (FILT && MODE == 1) {
    if (valid_q) {
      // sampling pass: items that fail the predicate do not count. The
      // predicate is evaluated into a bit mask first, so that every index into
      // r stays a compile-time constant and r stays in registers.
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        const uint32_t id0 = row0 + ch * 32;
        const uint32_t n_in = id0 >= static_cast<uint32_t>(p.N) ? 0u : min(32u, static_cast<uint32_t>(p.N) - id0);
        const uint32_t valid = n_in == 32 ? 0xffffffffu : ((1u << n_in) - 1u);
        uint32_t pm;
        if (use_sl) {
          pm = bloom_chunk_mask(sl + ch * 64, st) & valid;
        } else {
          pm = pred_pass_bits(p.filter, q, id0, valid, tile_rows, row0 - 32u * (chunk0 & 3));
        }
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (!((pm >> j) & 1u)) r[ch][j] = 0x7fc00000u;
        if (use_sl && p.filter.mode == kFilterBloomRecheck) {
          // Only the tile's best Bloom-passing item (the lowest index among equal scores) is
          // rechecked, once, after the tile's last chunk: the tile then counts that item if
          // it passes exactly, else nothing.
          const float mx = max32(r[ch]);
          if (mx > tb.sc || (tb.sc != tb.sc && mx == mx)) {
            uint32_t at = 0;
#pragma unroll
            for (int j = 0; j < 32; ++j) at |= static_cast<uint32_t>(__uint_as_float(r[ch][j]) == mx) << j;
            at &= pm;
            tb.sc = mx;
            tb.id = id0 + static_cast<uint32_t>(__ffs(at) - 1);
          }
          if (((chunk0 + ch) & 3) == 3) {
            bool ok = tb.sc == tb.sc;
            if (ok && wterms != nullptr) {
              const int ca = p.filter.C * p.filter.A;
              ok = pred_exact_row_sm(wterms + (threadIdx.x & 31) * kMaxTerms, ent,
                                     tile_rows + static_cast<size_t>(tb.id - (row0 + 32u * ch - 96u)) * ca, ca,
                                     p.filter.A);
            } else if (ok) {
              ok = pred_exact_item(p.filter, p.filter.terms + static_cast<size_t>(q) * kMaxTerms, p.filter.n_terms[q],
                                   tb.id, tile_rows, row0 + 32u * ch - 96u);
            }
            if (!ok) tb.sc = __uint_as_float(0x7fc00000u);
          }
        } else {
          // the tile's max over its passing items, chunk by chunk
          tb.sc = fmaxf(tb.sc, max32(r[ch]));
        }
      }
    }
  }
  if constexpr (MODE == 1) {
    // Sampling pass: one value per sampled tile, the max of its 128 scores (of its passing
    // items in the filtered variants: tb carries it over the tile's chunks). k sampled tiles
    // are k distinct items, so the k-th largest value is a lower bound on the k-th best score.
    if (valid_q) {
      float* dst = p.chunk_max + static_cast<size_t>(q) * p.chunk_stride;
      if constexpr (FILT) {
        if (((chunk0 + NCH - 1) & 3) == 3) {
          dst[(chunk0 + NCH - 1) >> 2] = tb.sc;
          tb.sc = __uint_as_float(0x7fc00000u);
        }
      } else {
        float m = -INFINITY;
        bool any = false;
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          const float c = max32(r[ch]);
          any |= c == c;
          m = fmaxf(m, c);
        }
        if (((chunk0 + NCH - 1) & 3) == 3) dst[(chunk0 + NCH - 1) >> 2] = any ? m : __uint_as_float(0x7fc00000u);
      }
    }
  } else {
    // Threshold filter: a chunk may hold a passing score iff its max (three-
    // input maxima, NaN ignored) is >= thresh; then the exact append of those
    // chunks, score by score.
    float cm[NCH];
    float all = -INFINITY;
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      // a chunk proved below the threshold: NaN, which passes no test and fmaxf ignores
      cm[ch] = ((live >> ch) & 1u) ? max32(r[ch]) : __uint_as_float(0x7fc00000u);
      all = fmaxf(all, cm[ch]);
    }
    if (__any_sync(RB_FULL_MASK, valid_q && all >= thresh)) {
      if constexpr (!FILT) {
        // the warp appends the chunks some lane may keep (stage: the upper half of the
        // warp's scratch; the int8 item scales use the lower half)
        uint32_t pass = 0;
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) pass |= static_cast<uint32_t>(valid_q && cm[ch] >= thresh) << ch;
        warp_append_chunks<NCH>(list, count, thresh, r, pass, row0, stage + 128);
      }
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        if constexpr (FILT) {
          // the lanes whose chunk max reached the threshold: each one's Bloom mask of the
          // chunk (32 items a term), then the warp tests and appends their items together
          const bool lp = valid_q && cm[ch] >= thresh;
          const uint32_t who = __ballot_sync(RB_FULL_MASK, lp);
          if (who != 0u) {
            const uint32_t id0 = row0 + ch * 32;
            const uint32_t bm = (lp && use_sl) ? bloom_chunk_mask(sl + ch * 64, st) : 0xffffffffu;
            if (__popc(who) <= kCoopFilterLanes) {
              warp_filter_append(p.filter, list, count, thresh, r[ch], who, bm, use_sl, q, id0, stage + 128,
                                 tile_rows, row0 - 32u * (chunk0 & 3), wterms, ent);
            } else {
              // many lanes at once (selective predicates, low thresholds): each lane tests its
              // own items, the predicate item by item only where some item is left
              uint32_t pm = lp ? (chunk_pass_bits(r[ch], thresh) & bm) : 0u;
              if (__any_sync(RB_FULL_MASK, pm != 0u)) {
                if (pm != 0u) {
                  const uint32_t tile0 = row0 - 32u * (chunk0 & 3);
                  if (!use_sl)
                    pm = pred_pass_bits(p.filter, q, id0, pm, tile_rows, tile0);
                  else if (p.filter.mode == kFilterBloomRecheck)
                    pm = pred_exact_bits(p.filter, q, id0, pm, tile_rows, tile0, wterms, ent);
                }
                if (pm != 0u) append_chunk_mask(list, count, r[ch], pm, id0);
              }
            }
          }
        }
      }
    }
  }
}

template <int MODE, int ELEM, int KB, int NG, int STAGES, int EPL, bool FILT>
__global__ void __launch_bounds__(64 + 128 * NG, 1)
    dense_scan_kernel(const __grid_constant__ DenseScanParams p) {
  using L = DenseSmemLayout<KB, NG, STAGES, FILT>;
  constexpr int kElemBytes = (ELEM == 2 || ELEM == 4) ? 1 : 2;
  constexpr int kElemsPerKBlock = 128 / kElemBytes;
  constexpr int kKSteps = 128 / 32;  // MMA K = 32 bytes per instruction
  constexpr uint32_t kTmemCols = 2 * NG * 128;
  constexpr uint32_t kIdesc =
      (ELEM == 2) ? make_idesc(2, 1, kQTile, kTileItems)
                  : make_idesc(1, ELEM == 1 ? 1 : 0, kQTile, kTileItems);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + L::kA;
  uint32_t* hist_all = reinterpret_cast<uint32_t*>(smem + L::kA + L::kB);
  uint32_t* slices_all = reinterpret_cast<uint32_t*>(smem + L::kA + L::kB + L::kHist);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kA + L::kB + L::kHist + L::kSlices);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* a_full = bars + 2 * STAGES;
  uint64_t* a_empty = a_full + 1;
  uint64_t* acc_full = a_full + 2;   // [2]
  uint64_t* acc_empty = a_full + 4;  // [2]
  uint64_t* drain_bar = a_full + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tasks = p.n_qsg * p.n_splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], L::kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmap_q);
    tma_prefetch_desc(&p.tmap_x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int a_iter = 0;
      uint32_t armed = 0;  // item stages armed in total
      for (int t = blockIdx.x; t < n_tasks && !*abort_flag; t += gridDim.x) {
        if (!task_live(p, t)) continue;  // every role skips the same tasks
        const int qsg = t % p.n_qsg, split = t / p.n_qsg;
        if (a_iter > 0 && !mbar_wait(a_empty, (a_iter - 1) & 1, abort_flag)) {
          atomicCAS(p.err, 0, kDevTimeoutProducer);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(a_full, NG * KB * L::kOpTile);
        for (int g = 0; g < NG; ++g)
          for (int kb = 0; kb < KB; ++kb)
            tma_load_2d(smA + (g * KB + kb) * L::kOpTile, &p.tmap_q, a_full, kb * kElemsPerKBlock,
                        qsg * NG * kQTile + g * kQTile);
        ++a_iter;
        int lo, hi;
        split_range(split, p.n_splits, p.pass_tiles, lo, hi);
        for (int pt = lo; pt < hi; ++pt) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag)) {
            atomicCAS(p.err, 0, kDevTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          const int tile = pt * p.tile_stride + p.tile_offset;
          mbar_arrive_expect_tx(&full_bar[stage], KB * L::kOpTile);
          for (int kb = 0; kb < KB; ++kb)
            tma_load_2d(smB + (stage * KB + kb) * L::kOpTile, &p.tmap_x, &full_bar[stage], kb * kElemsPerKBlock,
                        tile * kTileItems);
          ++armed;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every TMA this thread issued has landed before the CTA may exit.
      if (a_iter > 0) mbar_wait_drain(a_full, (a_iter - 1) & 1);
      for (int s = 0; s < STAGES; ++s) {
        const uint32_t n_s = armed / STAGES + (static_cast<uint32_t>(s) < armed % STAGES ? 1u : 0u);
        if (n_s > 0) mbar_wait_drain(&full_bar[s], (n_s - 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      int a_iter = 0;
      const uint32_t a_base = smem_u32(smA), b_base = smem_u32(smB);
      for (int t = blockIdx.x; t < n_tasks && !*abort_flag; t += gridDim.x) {
        if (!task_live(p, t)) continue;  // every role skips the same tasks
        const int split = t / p.n_qsg;
        if (!mbar_wait(a_full, a_iter & 1, abort_flag)) {
          atomicCAS(p.err, 0, kDevTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        ++a_iter;
        int lo, hi;
        split_range(split, p.n_splits, p.pass_tiles, lo, hi);
        bool ok = true;
        for (int pt = lo; pt < hi; ++pt) {
          if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag) ||
              !mbar_wait(&full_bar[stage], phase, abort_flag)) {
            atomicCAS(p.err, 0, kDevTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_col = tmem_base + static_cast<uint32_t>(acc * NG * 128);
#pragma unroll
          for (int g = 0; g < NG; ++g) {
#pragma unroll
            for (int kb = 0; kb < KB; ++kb) {
#pragma unroll
              for (int j = 0; j < kKSteps; ++j) {
                const uint64_t ad = sw128_kmajor_desc(a_base + (g * KB + kb) * L::kOpTile + j * 32);
                const uint64_t bd = sw128_kmajor_desc(b_base + (stage * KB + kb) * L::kOpTile + j * 32);
                if constexpr (ELEM == 2)
                  mma_i8(d_col + g * 128, ad, bd, kIdesc, (kb | j) != 0);
                else if constexpr (ELEM == 4)
                  mma_f8(d_col + g * 128, ad, bd, kIdesc, (kb | j) != 0);
                else
                  mma_f16(d_col + g * 128, ad, bd, kIdesc, (kb | j) != 0);
              }
            }
          }
          mma_commit(&empty_bar[stage]);
          mma_commit(&acc_full[acc]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1;
        }
        if (!ok) break;
        mma_commit(a_empty);
      }
      // Drain: no MMA may still be writing TMEM when it is released.
      mma_commit(drain_bar);
      mbar_wait_drain(drain_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;             // 0 .. 4*NG-1
    const int g = ew >> 2;               // query group
    const int quad = warp & 3;           // TMEM lane quadrant this warp may access
    uint32_t* hist = hist_all + ew * 256;
    // filtered variants: this warp's copies of the current and next tiles' bit-sliced Bloom words
    uint32_t* const sl_base = slices_all + ew * 2 * kTileSliceWords;
    const bool sliced = FILT && p.filter.slices != nullptr &&
                        (p.filter.mode == kFilterBloom || p.filter.mode == kFilterBloomRecheck);
    int acc = 0;
    uint32_t acc_phase = 0;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    for (int t = blockIdx.x; t < n_tasks; t += gridDim.x) {
      if (!task_live(p, t)) continue;  // every role skips the same tasks
      const int qsg = t % p.n_qsg, split = t / p.n_qsg;
      const int q = qsg * NG * kQTile + g * kQTile + quad * 32 + lane;
      const bool valid_q = q < p.B;
      float thresh = (valid_q && p.seed != nullptr) ? p.seed[q] : -INFINITY;
      int count = 0;
      // filtered variants: the query's Bloom terms for the bit-sliced test
      SlicedTerms st{};
      TileBest tb{__uint_as_float(0x7fc00000u), 0u};
      bool use_sl = false;
      if constexpr (FILT) {
        if (sliced) {
          st = load_sliced_terms(p.filter, q, valid_q);
          use_sl = valid_q && st.ok;
        }
      }
      uint2* list = p.lists + (static_cast<size_t>(valid_q ? q : 0) * p.n_splits + split) * p.cap;
      int lo, hi;
      split_range(split, p.n_splits, p.pass_tiles, lo, hi);
      bool ok = true;
      // int8: the item scales one tile ahead, the query's scale once per task
      ScalePrefetch sp_cur{}, sp_next{};
      if constexpr (ELEM == 2 && !FILT) {
        const float qsv = !valid_q ? 0.f : (p.q_scale != nullptr ? p.q_scale[q] : 1.f);
        sp_cur.qs = sp_next.qs = qsv;
        sp_cur.on = sp_next.on = true;
        if (lo < hi)
          sp_cur.xs = load_tile_scales(p, static_cast<uint32_t>((lo * p.tile_stride + p.tile_offset) * kTileItems));
      }
      for (int pt = lo; pt < hi; ++pt) {
        if constexpr (ELEM == 2 && !FILT) {
          if (pt + 1 < hi)
            sp_next.xs =
                load_tile_scales(p, static_cast<uint32_t>(((pt + 1) * p.tile_stride + p.tile_offset) * kTileItems));
        }
        if constexpr (MODE == 0) {
          // Room for a whole tile of appends; compacting here keeps no scores live
          // across the (non-inlined) compaction.
          const bool need = valid_q && (count > p.cap - kTileItems);
          if (__any_sync(RB_FULL_MASK, need)) warp_compact_lists<EPL>(list, count, thresh, need, p.k, hist);
        }
        if constexpr (FILT) {
          if (sliced) {
            // the next tile's slices (32 bytes a lane) land while this one is scanned; a
            // task's first tile is fetched here too
            __syncwarp();  // every lane is done with the buffer the next tile reuses
            if (pt == lo) {
              copy_tile_slices(sl_base, p, pt, lane);
              cp_async_commit();
            }
            if (pt + 1 < hi) copy_tile_slices(sl_base, p, pt + 1, lane);
            cp_async_commit();
          }
        }
        if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag)) {
          if (lane == 0) atomicCAS(p.err, 0, kDevTimeoutEpilogue);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t row0 = static_cast<uint32_t>((pt * p.tile_stride + p.tile_offset) * kTileItems);
        const uint32_t col0 = tmem_base + lane_addr + static_cast<uint32_t>(acc * NG * 128 + g * 128);
        uint32_t* const sl = sl_base + (pt & 1) * kTileSliceWords;
        // Unfiltered: the whole 128-column row in one go, then the accumulator goes
        // back to the MMA warp before any filtering work.
        if constexpr (FILT) {
          // One 32-item chunk at a time, TMEM as the staging: a single copy of the filtered
          // chunk code (four unrolled copies overflow the instruction cache), and 32 score
          // registers instead of 128.
          if (sliced) {
            cp_async_wait_group1();  // this tile's slices (the next tile's may still be in flight)
            __syncwarp();
          }
// Chunks to process (bit ch). The full pass first takes the tile's four chunk maxima
          // with all four loads in flight, and goes back to TMEM only for the chunks where some
          // lane's max reaches its threshold; the sampling pass evaluates every chunk.
          uint32_t todo = 0xfu;
          if constexpr (MODE == 0) {
            uint32_t r4[4][32];
            __syncwarp();
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) tmem_ld_32x32(col0 + ch * 32, r4[ch]);
            tmem_wait_ld();
            uint32_t mine = 0;
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) mine |= static_cast<uint32_t>(valid_q && max32(r4[ch]) >= thresh) << ch;
            todo = __reduce_or_sync(RB_FULL_MASK, mine);
          }
          if (todo == 0u) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
          }
          const int last = todo == 0u ? -1 : 31 - __clz(todo);
#pragma unroll 1
          for (int ch = 0; ch <= last; ++ch) {
            if (!((todo >> ch) & 1u)) continue;  // warp-uniform
            uint32_t r1[1][32];
            __syncwarp();
            tmem_ld_32x32(col0 + ch * 32, r1[0]);
            tmem_wait_ld();
            if (ch == last) {  // the accumulator goes back after the tile's last load
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&acc_empty[acc]);
            }
            process_chunks<MODE, 1, ELEM, FILT, KB>(p, r1, row0 + ch * 32, pt * 4 + ch, valid_q, q, thresh, count,
                                                    list, hist, sl + ch * 64, st, use_sl, tb);
          }
        } else {
          uint32_t r[4][32];
          __syncwarp();
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) tmem_ld_32x32(col0 + ch * 32, r[ch]);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[acc]);
          process_chunks<MODE, 4, ELEM, FILT, KB>(p, r, row0, pt * 4, valid_q, q, thresh, count, list, hist, sl, st,
                                                  use_sl, tb, nullptr, nullptr, 0, sp_cur);
          if constexpr (ELEM == 2 && !FILT) sp_cur = sp_next;
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      if (!ok) break;
      if constexpr (MODE == 0) {
        const bool need = valid_q && count > p.k;
        warp_compact_lists<EPL>(list, count, thresh, need, p.k, hist);
        if (valid_q) p.counts[static_cast<size_t>(q) * p.n_splits + split] = count;
      }
    }
  }

  if constexpr (FILT) cp_async_wait_all();  // slice copies of an early exit land before the CTA ends
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}


// ===========================================================================
// 2-SM variant: a CTA pair (cluster of 2) runs tcgen05.mma.cta_group::2 with
// M = 256 queries (128 per CTA) and N = 128 items (64 per CTA), NG query groups
// per pair. Per SM this halves the item bytes read from L2 for the same MMA
// work and cuts the operand bytes each MMA reads from shared memory, the two
// limits of the 1-SM kernel at large batches. CTA 0 of the pair issues the MMAs;
// both CTAs' TMA loads complete on CTA 0's barriers; CTA 0's commits reach both
// CTAs' barriers; the epilogue of each CTA reads its own TMEM rows and releases
// the accumulator with an arrive on CTA 0's barrier. No multicast anywhere.
// ===========================================================================
constexpr int kHalfItems = kTileItems / 2;

template <int KB, int NG, int STAGES, bool FILT = false>
struct Dense2SmLayout {
  static constexpr int kATile = kQTile * 128;     // 128 query rows x 128 bytes
  static constexpr int kBTile = kHalfItems * 128;  // 64 item rows x 128 bytes
  static constexpr int kA = NG * KB * kATile;
  static constexpr int kB = STAGES * KB * kBTile;
  static constexpr int kEpiWarps = 4 * NG;  // (group, lane quadrant)
  static constexpr int kHist = kEpiWarps * 256 * 4;
  // filtered variants: a ring of kRingSlots tiles, each its Bloom slices and attribute rows
  static constexpr int kRing = FILT ? kRingSlots * kRingSlotBytes : 0;
  // and each epilogue warp's table of its 32 queries' exact terms
  static constexpr int kTerms = FILT ? kEpiWarps * 32 * kMaxTerms * static_cast<int>(sizeof(ExactTerm)) : 0;
  static constexpr int kBar = (2 * STAGES + 2 + 2 * 4 + 1 + (FILT ? 2 * kRingSlots : 0)) * 8;
  static constexpr int kMisc = 16;
  static constexpr int kTotal = kA + kB + kHist + kRing + kTerms + kBar + kMisc + 1024;
};

template <int MODE, int ELEM, int KB, int NG, int STAGES, int EPL, bool FILT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(64 + 128 * NG, 1)
    dense_scan_2sm_kernel(const __grid_constant__ DenseScanParams p) {
  using L = Dense2SmLayout<KB, NG, STAGES, FILT>;
  constexpr int kElemBytes = (ELEM == 2 || ELEM == 4) ? 1 : 2;
  constexpr int kElemsPerKBlock = 128 / kElemBytes;
  constexpr int kKSteps = 128 / 32;
  constexpr int kAcc = 4 / NG;  // accumulator buffers: all 512 TMEM columns
  constexpr uint32_t kTmemCols = kAcc * NG * 128;
  constexpr uint32_t kIdesc = (ELEM == 2) ? make_idesc(2, 1, 2 * kQTile, kTileItems)
                                          : make_idesc(1, ELEM == 1 ? 1 : 0, 2 * kQTile, kTileItems);
  constexpr int kQPerPair = NG * 2 * kQTile;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + L::kA;
  uint32_t* hist_all = reinterpret_cast<uint32_t*>(smem + L::kA + L::kB);
  uint8_t* ring = smem + L::kA + L::kB + L::kHist;  // filtered variants
  ExactTerm* terms_all = reinterpret_cast<ExactTerm*>(smem + L::kA + L::kB + L::kHist + L::kRing);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kA + L::kB + L::kHist + L::kRing + L::kTerms);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* a_full = bars + 2 * STAGES;
  uint64_t* a_empty = a_full + 1;
  uint64_t* acc_full = a_full + 2;              // [kAcc][NG]
  uint64_t* acc_empty = acc_full + kAcc * NG;  // [kAcc][NG], used on CTA 0
  uint64_t* drain_bar = acc_empty + kAcc * NG;
  uint64_t* ring_full = drain_bar + 1;           // [kRingSlots] (filtered variants)
  uint64_t* ring_empty = ring_full + kRingSlots;  // [kRingSlots]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1 + (FILT ? 2 * kRingSlots : 0));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;
  const int n_tasks = p.n_qsg * p.n_splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int b = 0; b < kAcc * NG; ++b) {  // one pair per (buffer, query group): 4 warps a CTA each
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * 4);
    }
    mbar_init(drain_bar, 1);
    if constexpr (FILT) {
      for (int s = 0; s < kRingSlots; ++s) {
        mbar_init(&ring_full[s], 1);
        mbar_init(&ring_empty[s], L::kEpiWarps);
      }
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmap_q);
    tma_prefetch_desc(&p.tmap_x);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int a_iter = 0;
      uint32_t armed = 0;
      int rslot = 0;
      uint32_t rphase = 0, r_armed = 0;
      for (int t = pair; t < n_tasks && !*abort_flag; t += n_pairs) {
        if (!task_live(p, t)) continue;  // every role skips the same tasks
        const int qsg = t % p.n_qsg, split = t / p.n_qsg;
        if (a_iter > 0 && !mbar_wait(a_empty, (a_iter - 1) & 1, abort_flag)) {
          atomicCAS(p.err, 0, kDevTimeoutProducer);
          *abort_flag = 1;
          break;
        }
        if (rank == 0) mbar_arrive_expect_tx(a_full, 2 * NG * KB * L::kATile);
        for (int g = 0; g < NG; ++g)
          for (int kb = 0; kb < KB; ++kb)
            tma_load_2d_pair(smA + (g * KB + kb) * L::kATile, &p.tmap_q, a_full, kb * kElemsPerKBlock,
                             qsg * kQPerPair + g * 2 * kQTile + static_cast<int>(rank) * kQTile);
        ++a_iter;
        int lo, hi;
        split_range(split, p.n_splits, p.pass_tiles, lo, hi);
        for (int pt = lo; pt < hi; ++pt) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag)) {
            atomicCAS(p.err, 0, kDevTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          const int tile = pt * p.tile_stride + p.tile_offset;
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * KB * L::kBTile);
          for (int kb = 0; kb < KB; ++kb)
            tma_load_2d_pair(smB + (stage * KB + kb) * L::kBTile, &p.tmap_x, &full_bar[stage],
                             kb * kElemsPerKBlock, tile * kTileItems + static_cast<int>(rank) * kHalfItems);
          ++armed;
          if constexpr (FILT) {
            if (p.ring != 0) {
              // this CTA's copy of the tile's Bloom slices and attribute rows, once the
              // epilogue warps are done with the slot's previous tile
              if (!mbar_wait(&ring_empty[rslot], rphase ^ 1, abort_flag)) {
                atomicCAS(p.err, 0, kDevTimeoutProducer);
                *abort_flag = 1;
                break;
              }
              uint8_t* slot = ring + rslot * kRingSlotBytes;
              const int ca = p.filter.C * p.filter.A;
              const uint32_t n_in = static_cast<uint32_t>(min(kTileItems, p.N - tile * kTileItems));
              const uint32_t sl_bytes = (p.ring & 1) ? kTileSliceWords * 4u : 0u;
              const uint32_t row_bytes = (p.ring & 2) ? n_in * static_cast<uint32_t>(ca) * 8u : 0u;
              mbar_arrive_expect_tx(&ring_full[rslot], sl_bytes + row_bytes);
              if (sl_bytes != 0u)
                bulk_load(slot, p.filter.slices + static_cast<size_t>(tile) * kTileSliceWords, sl_bytes,
                          &ring_full[rslot]);
              if (row_bytes != 0u)
                bulk_load(slot + kTileSliceWords * 4,
                          p.filter.attrs + static_cast<size_t>(tile) * kTileItems * static_cast<size_t>(ca), row_bytes,
                          &ring_full[rslot]);
              ++r_armed;
              if (++rslot == kRingSlots) {
                rslot = 0;
                rphase ^= 1;
              }
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if constexpr (FILT) {  // this CTA's ring copies have landed
        for (int s = 0; s < kRingSlots; ++s) {
          const uint32_t n_s = r_armed / kRingSlots + (static_cast<uint32_t>(s) < r_armed % kRingSlots ? 1u : 0u);
          if (n_s > 0) mbar_wait_drain(&ring_full[s], (n_s - 1) & 1);
        }
      }
      // Drain (CTA 0's barriers count both CTAs' bytes): every load has landed.
      if (rank == 0) {
        if (a_iter > 0) mbar_wait_drain(a_full, (a_iter - 1) & 1);
        for (int s = 0; s < STAGES; ++s) {
          const uint32_t n_s = armed / STAGES + (static_cast<uint32_t>(s) < armed % STAGES ? 1u : 0u);
          if (n_s > 0) mbar_wait_drain(&full_bar[s], (n_s - 1) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (CTA 0)
    // The whole warp runs the loop on warp-uniform values; one elected lane
    // issues each tcgen05 instruction.
    if (rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      int a_iter = 0;
      const uint64_t a_desc0 = sw128_kmajor_desc(smem_u32(smA));
      const uint64_t b_desc0 = sw128_kmajor_desc(smem_u32(smB));
      const uint32_t empty0 = mapa_shared(smem_u32(empty_bar), 0), empty1 = mapa_shared(smem_u32(empty_bar), 1);
      const uint32_t accf0 = mapa_shared(smem_u32(acc_full), 0), accf1 = mapa_shared(smem_u32(acc_full), 1);
      const uint32_t ae0 = mapa_shared(smem_u32(a_empty), 0), ae1 = mapa_shared(smem_u32(a_empty), 1);
      for (int t = pair; t < n_tasks && !*abort_flag; t += n_pairs) {
        if (!task_live(p, t)) continue;  // every role skips the same tasks
        const int split = t / p.n_qsg;
        if (!__all_sync(RB_FULL_MASK, mbar_wait(a_full, a_iter & 1, abort_flag))) {
          if (lane == 0) atomicCAS(p.err, 0, kDevTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        ++a_iter;
        int lo, hi;
        split_range(split, p.n_splits, p.pass_tiles, lo, hi);
        bool ok = true;
        for (int pt = lo; pt < hi; ++pt) {
          if (!__all_sync(RB_FULL_MASK, mbar_wait(&full_bar[stage], phase, abort_flag))) {
            if (lane == 0) atomicCAS(p.err, 0, kDevTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          const uint32_t d_col = tmem_base + static_cast<uint32_t>(acc * NG * 128);
          const uint64_t b_stage = b_desc0 + static_cast<uint64_t>((stage * KB * L::kBTile) >> 4);
          // Each query group's MMAs go as soon as that group's epilogue warps have released
          // its accumulator, so one group's slow warp does not hold the other group back.
#pragma unroll
          for (int g = 0; g < NG; ++g) {
            if (!__all_sync(RB_FULL_MASK, mbar_wait(&acc_empty[acc * NG + g], acc_phase ^ 1, abort_flag))) {
              if (lane == 0) atomicCAS(p.err, 0, kDevTimeoutMma);
              *abort_flag = 1;
              ok = false;
              break;
            }
            tc_fence_after();
            if (elect_one()) {
#pragma unroll
              for (int kb = 0; kb < KB; ++kb) {
#pragma unroll
                for (int j = 0; j < kKSteps; ++j) {
                  const uint64_t ad = a_desc0 + static_cast<uint64_t>(((g * KB + kb) * L::kATile + j * 32) >> 4);
                  const uint64_t bd = b_stage + static_cast<uint64_t>((kb * L::kBTile + j * 32) >> 4);
                  if constexpr (ELEM == 2)
                    mma_i8_pair(d_col + g * 128, ad, bd, kIdesc, (kb | j) != 0);
                  else if constexpr (ELEM == 4)
                    mma_f8_pair(d_col + g * 128, ad, bd, kIdesc, (kb | j) != 0);
                  else
                    mma_f16_pair(d_col + g * 128, ad, bd, kIdesc, (kb | j) != 0);
                }
              }
              const uint32_t ao = static_cast<uint32_t>(acc * NG + g) * 8u;
              mma_commit_pair(accf0 + ao);
              mma_commit_pair(accf1 + ao);
            }
            __syncwarp();
          }
          if (!ok) break;
          if (elect_one()) {  // the item stage goes back once every group's MMAs are done with it
            const uint32_t so = static_cast<uint32_t>(stage) * 8u;
            mma_commit_pair(empty0 + so);
            mma_commit_pair(empty1 + so);
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          if (++acc == kAcc) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
        if (!ok) break;
        if (elect_one()) {
          mma_commit_pair(ae0);
          mma_commit_pair(ae1);
        }
        __syncwarp();
      }
      if (elect_one()) mma_commit_pair(mapa_shared(smem_u32(drain_bar), 0));
      __syncwarp();
      mbar_wait_drain(drain_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    // Warp (group g, lane quadrant): its 32 queries x the group's 128 item
    // columns per step.
    const int ew = warp - 2;
    const int g = ew >> 2;
    const int quad = warp & 3;
    uint32_t* hist = hist_all + ew * 256;
    // filtered variants: the tile's Bloom slices (and attribute rows) from the ring
    const bool sliced = FILT && (p.ring & 1) != 0;
    // with the attribute rows in the ring: this warp's table of its queries' exact terms
    ExactTerm* const wterms = (FILT && (p.ring & 2) != 0) ? terms_all + ew * 32 * kMaxTerms : nullptr;
    int rslot = 0;
    uint32_t rphase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t release0 = mapa_shared(smem_u32(acc_empty), 0);
    for (int t = pair; t < n_tasks; t += n_pairs) {
      if (!task_live(p, t)) continue;  // every role skips the same tasks
      const int qsg = t % p.n_qsg, split = t / p.n_qsg;
      const int q = qsg * kQPerPair + g * 2 * kQTile + static_cast<int>(rank) * kQTile + quad * 32 + lane;
      const bool valid_q = q < p.B;
      float thresh = (valid_q && p.seed != nullptr) ? p.seed[q] : -INFINITY;
      int count = 0;
      // filtered variants: the query's Bloom terms for the bit-sliced test
      SlicedTerms st{};
      TileBest tb{__uint_as_float(0x7fc00000u), 0u};
      bool use_sl = false;
      int ent = 0;
      if constexpr (FILT) {
        if (sliced) {
          st = load_sliced_terms(p.filter, q, valid_q);
          use_sl = valid_q && st.ok;
        }
        if (wterms != nullptr) {
          __syncwarp();  // every lane is done with the previous task's table
          ent = valid_q ? min(p.filter.n_terms[q], kMaxTerms) : 0;
          const PredTerm* tq = p.filter.terms + static_cast<size_t>(valid_q ? q : 0) * kMaxTerms;
#pragma unroll 1
          for (int i = 0; i < kMaxTerms; ++i) {
            ExactTerm et{0, 0, 0};
            if (i < ent) {
              const PredTerm t = tq[i];
              et = ExactTerm{t.value, t.clause * p.filter.A, t.flags};
            }
            wterms[lane * kMaxTerms + i] = et;
          }
          __syncwarp();
        }
      }
      const size_t list_id = static_cast<size_t>(valid_q ? q : 0) * p.n_splits + split;
      uint2* list = p.lists + list_id * p.cap;
      int lo, hi;
      split_range(split, p.n_splits, p.pass_tiles, lo, hi);
      bool ok = true;
      // int8: the item scales one tile ahead, the query's scale once per task
      ScalePrefetch sp_cur{}, sp_next{};
      if constexpr (ELEM == 2 && !FILT) {
        const float qsv = !valid_q ? 0.f : (p.q_scale != nullptr ? p.q_scale[q] : 1.f);
        sp_cur.qs = sp_next.qs = qsv;
        sp_cur.on = sp_next.on = true;
        if (lo < hi)
          sp_cur.xs = load_tile_scales(p, static_cast<uint32_t>((lo * p.tile_stride + p.tile_offset) * kTileItems));
      }
      for (int pt = lo; pt < hi; ++pt) {
        if constexpr (ELEM == 2 && !FILT) {
          if (pt + 1 < hi)
            sp_next.xs =
                load_tile_scales(p, static_cast<uint32_t>(((pt + 1) * p.tile_stride + p.tile_offset) * kTileItems));
        }
        if constexpr (MODE == 0) {
          const bool need = valid_q && (count > p.cap - kTileItems);
          if (__any_sync(RB_FULL_MASK, need)) warp_compact_lists<EPL>(list, count, thresh, need, p.k, hist);
        }
        if (!mbar_wait(&acc_full[acc * NG + g], acc_phase, abort_flag)) {
          if (lane == 0) atomicCAS(p.err, 0, kDevTimeoutEpilogue);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t row0 = static_cast<uint32_t>((pt * p.tile_stride + p.tile_offset) * kTileItems);
        const uint32_t col0 = tmem_base + lane_addr + static_cast<uint32_t>(acc * NG * 128 + g * 128);
        const uint32_t* sl = nullptr;
        const int64_t* tile_rows = nullptr;
        if constexpr (FILT) {
          if (p.ring != 0) {
            if (!mbar_wait(&ring_full[rslot], rphase, abort_flag)) {
              if (lane == 0) atomicCAS(p.err, 0, kDevTimeoutEpilogue);
              *abort_flag = 1;
              ok = false;
              break;
            }
            const uint8_t* slot = ring + rslot * kRingSlotBytes;
            sl = reinterpret_cast<const uint32_t*>(slot);
            if (p.ring & 2) tile_rows = reinterpret_cast<const int64_t*>(slot + kTileSliceWords * 4);
          }
        }
        if constexpr (FILT) {
          // One 32-item chunk at a time, TMEM as the staging: a single copy of the filtered
          // chunk code (four unrolled copies overflow the instruction cache), and 32 score
          // registers instead of 128.
// Chunks to process (bit ch). The full pass first takes the tile's four chunk maxima
          // with all four loads in flight, and goes back to TMEM only for the chunks where some
          // lane's max reaches its threshold; the sampling pass evaluates every chunk.
          uint32_t todo = 0xfu;
          if constexpr (MODE == 0) {
            uint32_t r4[4][32];
            __syncwarp();
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) tmem_ld_32x32(col0 + ch * 32, r4[ch]);
            tmem_wait_ld();
            uint32_t mine = 0;
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) mine |= static_cast<uint32_t>(valid_q && max32(r4[ch]) >= thresh) << ch;
            todo = __reduce_or_sync(RB_FULL_MASK, mine);
          }
          if (todo == 0u) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(release0 + static_cast<uint32_t>(acc * NG + g) * 8u);
          }
          const int last = todo == 0u ? -1 : 31 - __clz(todo);
#pragma unroll 1
          for (int ch = 0; ch <= last; ++ch) {
            if (!((todo >> ch) & 1u)) continue;  // warp-uniform
            uint32_t r1[1][32];
            __syncwarp();
            tmem_ld_32x32(col0 + ch * 32, r1[0]);
            tmem_wait_ld();
            if (ch == last) {  // the accumulator goes back after the tile's last load
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster(release0 + static_cast<uint32_t>(acc * NG + g) * 8u);
            }
            process_chunks<MODE, 1, ELEM, FILT, KB>(p, r1, row0 + ch * 32, pt * 4 + ch, valid_q, q, thresh, count,
                                                    list, hist, sl + ch * 64, st, use_sl, tb, tile_rows, wterms,
                                                    ent);
          }
          if (p.ring != 0) {  // the slot goes back once every lane is done with it
            __syncwarp();
            if (lane == 0) mbar_arrive(&ring_empty[rslot]);
            if (++rslot == kRingSlots) {
              rslot = 0;
              rphase ^= 1;
            }
          }
        } else {
          uint32_t r[4][32];
          __syncwarp();
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) tmem_ld_32x32(col0 + ch * 32, r[ch]);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(release0 + static_cast<uint32_t>(acc * NG + g) * 8u);
          process_chunks<MODE, 4, ELEM, FILT, KB>(p, r, row0, pt * 4, valid_q, q, thresh, count, list, hist, sl, st,
                                                  use_sl, tb, nullptr, nullptr, 0, sp_cur);
          if constexpr (ELEM == 2 && !FILT) sp_cur = sp_next;
        }
        if (++acc == kAcc) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok) break;
      if constexpr (MODE == 0) {
        const bool need = valid_q && count > p.k;
        warp_compact_lists<EPL>(list, count, thresh, need, p.k, hist);
        if (valid_q) p.counts[list_id] = count;
      }
    }
  }

  __syncwarp();
  if (*abort_flag) {
    // Error path only: a load of this CTA may still be in flight towards its
    // own shared memory while it can no longer be tracked; let it land.
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) __nanosleep(10000);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal or read it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <int MODE, int ELEM, int KB, int NG, int STAGES, int EPL, bool FILT>
static cudaError_t launch_dense_scan(const DenseScanParams& prm, int grid, cudaStream_t stream) {
  using L = DenseSmemLayout<KB, NG, STAGES, FILT>;
  static_assert(L::kTotal <= kMaxSmemPerCta, "1-SM scan variant exceeds the shared memory of one CTA");
  auto kern = dense_scan_kernel<MODE, ELEM, KB, NG, STAGES, EPL, FILT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return e;
  }
  kern<<<grid, 64 + 128 * NG, L::kTotal, stream>>>(prm);
  return cudaGetLastError();
}

template <int MODE, int ELEM, int KB, int NG, int STAGES, int EPL, bool FILT>
static cudaError_t launch_dense_scan_2sm(const DenseScanParams& prm, int n_pairs, cudaStream_t stream) {
  using L = Dense2SmLayout<KB, NG, STAGES, FILT>;
  static_assert(L::kTotal <= kMaxSmemPerCta, "2-SM scan variant exceeds the shared memory of one CTA");
  auto kern = dense_scan_2sm_kernel<MODE, ELEM, KB, NG, STAGES, EPL, FILT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  if (e != cudaSuccess) {
    cudaGetLastError();  // the attribute's error is reported by the return value, not left pending
    return e;
  }
  kern<<<2 * n_pairs, 64 + 128 * NG, L::kTotal, stream>>>(prm);
  return cudaGetLastError();
}

// Picks the kernel for a pass: MODE 1 (sampling) or MODE 0 with the list
// compaction's entries per lane (40 only in one-group kernels, and not with
// attribute filters, whose lists stay within 512 entries).
template <int ELEM, int KB, int NG, int ST, bool F>
static cudaError_t launch_2sm_variant(int mode, int epl, const DenseScanParams& prm, int n_pairs,
                                      cudaStream_t stream) {
  if (mode == 1) return launch_dense_scan_2sm<1, ELEM, KB, NG, ST, 8, F>(prm, n_pairs, stream);
  if (epl == 8) return launch_dense_scan_2sm<0, ELEM, KB, NG, ST, 8, F>(prm, n_pairs, stream);
  if (epl == 16) return launch_dense_scan_2sm<0, ELEM, KB, NG, ST, 16, F>(prm, n_pairs, stream);
  if constexpr (NG == 1 && !F) return launch_dense_scan_2sm<0, ELEM, KB, NG, ST, 40, F>(prm, n_pairs, stream);
  return cudaErrorInvalidConfiguration;
}

template <int ELEM, int KB, int NG, int ST, bool F>
static cudaError_t launch_1sm_variant(int mode, int epl, const DenseScanParams& prm, int grid, cudaStream_t stream) {
  if (mode == 1) return launch_dense_scan<1, ELEM, KB, NG, ST, 8, F>(prm, grid, stream);
  if (epl == 8) return launch_dense_scan<0, ELEM, KB, NG, ST, 8, F>(prm, grid, stream);
  if (epl == 16) return launch_dense_scan<0, ELEM, KB, NG, ST, 16, F>(prm, grid, stream);
  if constexpr (NG == 1 && !F) return launch_dense_scan<0, ELEM, KB, NG, ST, 40, F>(prm, grid, stream);
  return cudaErrorInvalidConfiguration;
}

// CTA pairs of the 2-SM kernel that fit on the device at once (dense_scan_e1.cu).
int dense_max_pairs();

// 2-D K-major tensor map over rows x cols elements (elem: 0 fp16, 1 bf16, 2 / 4
// one-byte codes), boxes of box_rows x 128 bytes, 128-byte swizzle.
bool make_tmap_2d(CUtensorMap* map, const void* base, int elem, uint64_t rows, uint64_t cols, int box_rows);

// Launches the pass for one element type; false if no variant matches.
bool dense_launch_e0(bool two_sm, int mode, int kb, int ng, bool filtered, int epl, const DenseScanParams& prm,
                     int grid, cudaStream_t stream, cudaError_t& e);
bool dense_launch_e1(bool two_sm, int mode, int kb, int ng, bool filtered, int epl, const DenseScanParams& prm,
                     int grid, cudaStream_t stream, cudaError_t& e);
bool dense_launch_e2(bool two_sm, int mode, int kb, int ng, bool filtered, int epl, const DenseScanParams& prm,
                     int grid, cudaStream_t stream, cudaError_t& e);
bool dense_launch_e4(bool two_sm, int mode, int kb, int ng, bool filtered, int epl, const DenseScanParams& prm,
                     int grid, cudaStream_t stream, cudaError_t& e);

}  // namespace rb
