// Fused dense scoring + exact top-k for sm_100a (B200).
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
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "rb_capi_internal.h"
#include "rb_common.cuh"
#include "rb_select.cuh"

namespace rb {

constexpr int kTileItems = 128;  // N of one MMA = items per pipeline stage
constexpr int kQTile = 128;      // M of one MMA = queries per group
constexpr int kSampleStride = 16;  // sampling pass: every 16th tile

struct alignas(64) DenseScanParams {
  CUtensorMap tmap_q;
  CUtensorMap tmap_x;   // item boxes of 128 rows (1-SM kernel) or 64 rows (2-SM kernel)
  const float* seed;  // [B] pass threshold per query (>=), or null for -inf
  uint2* lists;       // [B, n_splits, cap]
  int* counts;        // [B, n_splits]
  int* err;           // device error word
  float* chunk_max;   // MODE 1: [B, chunk_stride] max score of every 32-item chunk
  int chunk_stride;
  const float* q_scale;  // int8 only: [B] per-query scale
  const float* x_scale;  // int8 only: [N] per-item scale
  FilterArgs filter;     // attribute predicate (mode kFilterNone: none)
  int B, N;
  int n_qsg, n_splits;
  int tile_stride, tile_offset, pass_tiles;
  int k, cap;
};

template <int KB, int NG, int STAGES>
struct DenseSmemLayout {
  static constexpr int kOpTile = kQTile * 128;  // bytes of one 128-row x 128-byte K-block
  static constexpr int kA = NG * KB * kOpTile;
  static constexpr int kB = STAGES * KB * kOpTile;
  static constexpr int kEpiWarps = 4 * NG;
  static constexpr int kHist = kEpiWarps * 256 * 4;
  static constexpr int kBar = (2 * STAGES + 2 + 4 + 1) * 8;
  static constexpr int kMisc = 16;
  static constexpr int kTotal = kA + kB + kHist + kBar + kMisc + 1024;  // + alignment slack
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
// For int8 (ELEM 2) the registers first hold int32 dots, turned here into the
// exact fp32 score (fp32(dot) * q_scale) * item_scale, left to right as the
// reference dequantizes (ops/official/adapter.py:338-367).
template <int MODE, int NCH, int ELEM, bool FILT, int KB>
__device__ __forceinline__ void process_chunks(const DenseScanParams& p, uint32_t (&r)[NCH][32], uint32_t row0,
                                               int chunk0, bool valid_q, int q, float thresh, int& count,
                                               uint2* list) {
  if constexpr (ELEM == 2) {
    // null scale arrays mean unit scales (the score is then the raw dot)
    const float qs = !valid_q ? 0.f : (p.q_scale != nullptr ? p.q_scale[q] : 1.f);
    const bool full = row0 + NCH * 32 <= static_cast<uint32_t>(p.N);
    const bool unit_x = p.x_scale == nullptr;
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const uint32_t id = row0 + ch * 32 + 4 * j4;
        float4 xs;
        if (unit_x) {
          xs = make_float4(1.f, 1.f, 1.f, 1.f);
        } else if (full) {
          xs = __ldg(reinterpret_cast<const float4*>(p.x_scale + id));
        } else {
          xs.x = id < static_cast<uint32_t>(p.N) ? p.x_scale[id] : 0.f;
          xs.y = id + 1 < static_cast<uint32_t>(p.N) ? p.x_scale[id + 1] : 0.f;
          xs.z = id + 2 < static_cast<uint32_t>(p.N) ? p.x_scale[id + 2] : 0.f;
          xs.w = id + 3 < static_cast<uint32_t>(p.N) ? p.x_scale[id + 3] : 0.f;
        }
        const float xv[4] = {xs.x, xs.y, xs.z, xs.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          // |dot| <= 2^22 for D <= 256: exact int32 -> fp32 through the fp32 magic
          // constant; D = 512 reaches 2^23, still exact in fp32 (< 2^24) by conversion
          float f;
          if constexpr (KB <= 2)
            f = __uint_as_float(r[ch][4 * j4 + u] + 0x4B400000u) - 12582912.0f;
          else
            f = __int2float_rn(static_cast<int>(r[ch][4 * j4 + u]));
          r[ch][4 * j4 + u] = __float_as_uint(__fmul_rn(__fmul_rn(f, qs), xv[u]));
        }
      }
    }
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
        const uint32_t pm = pred_pass_bits(p.filter, q, id0, valid);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (!((pm >> j) & 1u)) r[ch][j] = 0x7fc00000u;
      }
    }
  }
  if constexpr (MODE == 1) {
    // sampling pass: the max of every 32-item chunk, nothing else
    if (valid_q) {
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch)
        p.chunk_max[static_cast<size_t>(q) * p.chunk_stride + chunk0 + ch] = max32(r[ch]);
    }
  } else {
    // Threshold filter on the FMA pipe (paired fp32 subtracts) and the ALU
    // (AND tree): the sign bit of sg[ch] is set iff no score of chunk ch
    // passes; then the exact append of the chunks that may pass.
    const uint64_t tt = pack_pair(thresh);
    uint32_t sg[NCH];
    uint32_t all = 0xffffffffu;
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      sg[ch] = chunk_all_below(r[ch], tt);
      all &= sg[ch];
    }
    if (__any_sync(RB_FULL_MASK, valid_q && !(all >> 31))) {
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        if (valid_q && !(sg[ch] >> 31)) {
          if constexpr (!FILT) {
            append_chunk_bits(list, count, thresh, r[ch], row0 + ch * 32);
          } else {
            const uint32_t id0 = row0 + ch * 32;
            const uint32_t pm = pred_pass_bits(p.filter, q, id0, chunk_pass_bits(r[ch], thresh));
            append_chunk_mask(list, count, r[ch], pm, id0);
          }
        }
      }
    }
  }
}

template <int MODE, int ELEM, int KB, int NG, int STAGES, int EPL, bool FILT>
__global__ void __launch_bounds__(64 + 128 * NG, 1)
    dense_scan_kernel(const __grid_constant__ DenseScanParams p) {
  using L = DenseSmemLayout<KB, NG, STAGES>;
  constexpr int kElemBytes = (ELEM == 2) ? 1 : 2;
  constexpr int kElemsPerKBlock = 128 / kElemBytes;
  constexpr int kKSteps = 128 / 32;  // MMA K = 32 bytes per instruction
  constexpr uint32_t kTmemCols = 2 * NG * 128;
  constexpr uint32_t kIdesc =
      (ELEM == 2) ? make_idesc(2, 1, kQTile, kTileItems) : make_idesc(1, ELEM == 1 ? 1 : 0, kQTile, kTileItems);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + L::kA;
  uint32_t* hist_all = reinterpret_cast<uint32_t*>(smem + L::kA + L::kB);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kA + L::kB + L::kHist);
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
    int acc = 0;
    uint32_t acc_phase = 0;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    for (int t = blockIdx.x; t < n_tasks; t += gridDim.x) {
      const int qsg = t % p.n_qsg, split = t / p.n_qsg;
      const int q = qsg * NG * kQTile + g * kQTile + quad * 32 + lane;
      const bool valid_q = q < p.B;
      float thresh = (valid_q && p.seed != nullptr) ? p.seed[q] : -INFINITY;
      int count = 0;
      uint2* list = p.lists + (static_cast<size_t>(valid_q ? q : 0) * p.n_splits + split) * p.cap;
      int lo, hi;
      split_range(split, p.n_splits, p.pass_tiles, lo, hi);
      bool ok = true;
      for (int pt = lo; pt < hi; ++pt) {
        if constexpr (MODE == 0) {
          // Room for a whole tile of appends; compacting here keeps no scores live
          // across the (non-inlined) compaction.
          const bool need = valid_q && (count > p.cap - kTileItems);
          if (__any_sync(RB_FULL_MASK, need)) warp_compact_lists<EPL>(list, count, thresh, need, p.k, hist);
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
        // The whole 128-column row in one go, then the accumulator goes back to
        // the MMA warp before any filtering work.
        uint32_t r[4][32];
        __syncwarp();
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) tmem_ld_32x32(col0 + ch * 32, r[ch]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        process_chunks<MODE, 4, ELEM, FILT, KB>(p, r, row0, pt * 4, valid_q, q, thresh, count, list);
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

template <int KB, int NG, int STAGES>
struct Dense2SmLayout {
  static constexpr int kATile = kQTile * 128;     // 128 query rows x 128 bytes
  static constexpr int kBTile = kHalfItems * 128;  // 64 item rows x 128 bytes
  static constexpr int kA = NG * KB * kATile;
  static constexpr int kB = STAGES * KB * kBTile;
  static constexpr int kEpiWarps = 4 * NG;  // (group, lane quadrant)
  static constexpr int kHist = kEpiWarps * 256 * 4;
  static constexpr int kBar = (2 * STAGES + 2 + 2 * 4 + 1) * 8;
  static constexpr int kMisc = 16;
  static constexpr int kTotal = kA + kB + kHist + kBar + kMisc + 1024;
};

template <int MODE, int ELEM, int KB, int NG, int STAGES, int EPL, bool FILT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(64 + 128 * NG, 1)
    dense_scan_2sm_kernel(const __grid_constant__ DenseScanParams p) {
  using L = Dense2SmLayout<KB, NG, STAGES>;
  constexpr int kElemBytes = (ELEM == 2) ? 1 : 2;
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
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kA + L::kB + L::kHist);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* a_full = bars + 2 * STAGES;
  uint64_t* a_empty = a_full + 1;
  uint64_t* acc_full = a_full + 2;         // [kAcc]
  uint64_t* acc_empty = acc_full + kAcc;  // [kAcc], used on CTA 0
  uint64_t* drain_bar = acc_empty + kAcc;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
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
    for (int b = 0; b < kAcc; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * L::kEpiWarps);
    }
    mbar_init(drain_bar, 1);
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
      for (int t = pair; t < n_tasks && !*abort_flag; t += n_pairs) {
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
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
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
          const bool ready = mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag) &&
                             mbar_wait(&full_bar[stage], phase, abort_flag);
          if (!__all_sync(RB_FULL_MASK, ready)) {
            if (lane == 0) atomicCAS(p.err, 0, kDevTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_col = tmem_base + static_cast<uint32_t>(acc * NG * 128);
          const uint64_t b_stage = b_desc0 + static_cast<uint64_t>((stage * KB * L::kBTile) >> 4);
          if (elect_one()) {
#pragma unroll
            for (int g = 0; g < NG; ++g) {
#pragma unroll
              for (int kb = 0; kb < KB; ++kb) {
#pragma unroll
                for (int j = 0; j < kKSteps; ++j) {
                  const uint64_t ad = a_desc0 + static_cast<uint64_t>(((g * KB + kb) * L::kATile + j * 32) >> 4);
                  const uint64_t bd = b_stage + static_cast<uint64_t>((kb * L::kBTile + j * 32) >> 4);
                  if constexpr (ELEM == 2)
                    mma_i8_pair(d_col + g * 128, ad, bd, kIdesc, (kb | j) != 0);
                  else
                    mma_f16_pair(d_col + g * 128, ad, bd, kIdesc, (kb | j) != 0);
                }
              }
            }
            const uint32_t so = static_cast<uint32_t>(stage) * 8u, ao = static_cast<uint32_t>(acc) * 8u;
            mma_commit_pair(empty0 + so);
            mma_commit_pair(empty1 + so);
            mma_commit_pair(accf0 + ao);
            mma_commit_pair(accf1 + ao);
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
    int acc = 0;
    uint32_t acc_phase = 0;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t release0 = mapa_shared(smem_u32(acc_empty), 0);
    for (int t = pair; t < n_tasks; t += n_pairs) {
      const int qsg = t % p.n_qsg, split = t / p.n_qsg;
      const int q = qsg * kQPerPair + g * 2 * kQTile + static_cast<int>(rank) * kQTile + quad * 32 + lane;
      const bool valid_q = q < p.B;
      float thresh = (valid_q && p.seed != nullptr) ? p.seed[q] : -INFINITY;
      int count = 0;
      const size_t list_id = static_cast<size_t>(valid_q ? q : 0) * p.n_splits + split;
      uint2* list = p.lists + list_id * p.cap;
      int lo, hi;
      split_range(split, p.n_splits, p.pass_tiles, lo, hi);
      bool ok = true;
      for (int pt = lo; pt < hi; ++pt) {
        if constexpr (MODE == 0) {
          const bool need = valid_q && (count > p.cap - kTileItems);
          if (__any_sync(RB_FULL_MASK, need)) warp_compact_lists<EPL>(list, count, thresh, need, p.k, hist);
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
        uint32_t r[4][32];
        __syncwarp();
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) tmem_ld_32x32(col0 + ch * 32, r[ch]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(release0 + static_cast<uint32_t>(acc) * 8u);
        process_chunks<MODE, 4, ELEM, FILT, KB>(p, r, row0, pt * 4, valid_q, q, thresh, count, list);
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

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) == cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D K-major tensor map: rows x cols elements, box box_rows x 128 bytes, 128-B swizzle.
static bool make_tmap(CUtensorMap* map, const void* base, int elem, uint64_t rows, uint64_t cols, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const int eb = (elem == 2) ? 1 : 2;
  CUtensorMapDataType dt = (elem == 2)   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                           : (elem == 1) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * eb};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / eb), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int MODE, int ELEM, int KB, int NG, int STAGES, int EPL, bool FILT>
static cudaError_t launch_dense_scan(const DenseScanParams& prm, int grid, cudaStream_t stream) {
  using L = DenseSmemLayout<KB, NG, STAGES>;
  auto kern = dense_scan_kernel<MODE, ELEM, KB, NG, STAGES, EPL, FILT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  if (e != cudaSuccess) return e;
  kern<<<grid, 64 + 128 * NG, L::kTotal, stream>>>(prm);
  return cudaGetLastError();
}

template <int MODE, int ELEM, int KB, int NG, int STAGES, int EPL, bool FILT>
static cudaError_t launch_dense_scan_2sm(const DenseScanParams& prm, int n_pairs, cudaStream_t stream) {
  using L = Dense2SmLayout<KB, NG, STAGES>;
  auto kern = dense_scan_2sm_kernel<MODE, ELEM, KB, NG, STAGES, EPL, FILT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  if (e != cudaSuccess) return e;
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

// CTA pairs of the 2-SM kernel that fit on the device at once.
static int max_pairs() {
  static int n = 0;
  if (n == 0) {
    using L = Dense2SmLayout<2, 2, 8>;
    auto kern = dense_scan_2sm_kernel<0, 1, 2, 2, 8, 16, false>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74, 1, 1);
    cfg.blockDim = dim3(64 + 128 * 2, 1, 1);
    cfg.dynamicSmemBytes = L::kTotal;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
      cudaGetLastError();
      clusters = num_sms() / 2;
    }
    n = std::min(clusters, num_sms() / 2);
  }
  return n;
}

}  // namespace rb

// ---------------------------------------------------------------------------
// Scan-plan shared by the dense entry points.
// ---------------------------------------------------------------------------
namespace rb {

int list_cap(int k) {
  // room for k survivors + one 128-item tile of appends; multiple of 32
  return ((k + 128) + 31) / 32 * 32;
}

// Entries per lane of the register-resident list compaction for a list of cap.
static int dense_epl(int cap) { return cap <= 256 ? 8 : (cap <= 512 ? 16 : 40); }

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

void dense_plan(int B, int N, int k, int row_bytes, DensePlan& pl, int64_t n_total) {
  // B > 128: 2-SM kernel, 256 queries per group, 1 or 2 groups per CTA pair
  // (one for 512-byte rows, whose operand tiles fill shared memory, and for
  // lists past 512 entries, whose compaction needs the registers of a
  // 6-warp CTA).
  pl.two_sm = B > kQTile;
  if (pl.two_sm) {
    pl.ng = (B <= 2 * kQTile || row_bytes > 256 || list_cap(k) > 512) ? 1 : 2;
    pl.n_qsg = (B + pl.ng * 2 * kQTile - 1) / (pl.ng * 2 * kQTile);
    pl.n_splits = std::max(1, max_pairs() / pl.n_qsg);
    pl.n_lists = pl.n_splits;
  } else {
    pl.ng = 1;
    pl.n_qsg = 1;
    pl.n_splits = num_sms();
    pl.n_lists = pl.n_splits;
  }
  pl.cap = list_cap(k);
  pl.tiles = (N + kTileItems - 1) / kTileItems;
  // Optional sampling pass over every s-th tile: it records the max of each
  // 32-item chunk; the k-th largest chunk max is a lower bound on the k-th best
  // score of the corpus (k distinct items reach it) and seeds the full pass.
  // That bound sits near rank k * s of the corpus, so the full pass appends
  // about k * s candidates per query: s is the sparsest stride (at most
  // kSampleStride) that keeps those at no more than 0.1 per query row and
  // 128-item tile (over a corpus of n_total items: the union of every shard's
  // sample when the seed is shared) and still samples at least 4k chunks.
  pl.sample_stride = 0;
  const int64_t n_scale = std::max<int64_t>(n_total, N);
  for (int s = kSampleStride; s >= 1; s >>= 1) {
    const int64_t chunks = (pl.tiles + s - 1) / s * 4;
    const bool dense_enough = static_cast<double>(k) * s * kTileItems <= 0.1 * static_cast<double>(n_scale);
    if (chunks >= 4 * static_cast<int64_t>(k) && (dense_enough || s == 1)) {
      pl.sample_stride = s;
      break;
    }
  }
}

size_t dense_chunk_stride(const DensePlan& pl) {
  if (pl.sample_stride == 0) return 0;
  return static_cast<size_t>((pl.tiles + pl.sample_stride - 1) / pl.sample_stride) * 4;
}

size_t dense_workspace_bytes(int B, int N, int k, int row_bytes) {
  DensePlan pl;
  dense_plan(B, N, k, row_bytes, pl, N);
  size_t lists = static_cast<size_t>(B) * pl.n_lists * pl.cap * sizeof(uint2);
  size_t counts = static_cast<size_t>(B) * pl.n_lists * sizeof(int);
  size_t th = 2 * static_cast<size_t>(B) * sizeof(float);
  size_t cm = static_cast<size_t>(B) * dense_chunk_stride(pl) * sizeof(float);
  // the chunk maxima are dead once the seed is known: they share the list space
  return align_up(std::max(lists, cm), 256) + align_up(counts, 256) + align_up(th, 256) + 256;
}

int dense_scan_pass(int mode, int elem, const void* q, const void* x, int B, int N, int D, const DensePlan& pl,
                    int k, const float* seed, uint2* lists, int* counts, float* chunk_max, int* err,
                    cudaStream_t stream, const float* q_scale, const float* x_scale, const FilterArgs* filter) {
  DenseScanParams prm;
  std::memset(&prm, 0, sizeof(prm));
  const bool filtered = filter != nullptr && filter->mode != kFilterNone;
  if (filtered) prm.filter = *filter;
  prm.q_scale = q_scale;
  prm.x_scale = x_scale;
  const int eb = (elem == 2) ? 1 : 2;
  const int row_bytes = D * eb;
  const int item_box = pl.two_sm ? kHalfItems : kTileItems;
  if (!make_tmap(&prm.tmap_q, q, elem, static_cast<uint64_t>(B), static_cast<uint64_t>(D), kQTile) ||
      !make_tmap(&prm.tmap_x, x, elem, static_cast<uint64_t>(N), static_cast<uint64_t>(D), item_box)) {
    set_last_error("cuTensorMapEncodeTiled failed (alignment or driver entry point)");
    return RB_ERR_CUDA;
  }
  const int stride = (mode == 1) ? pl.sample_stride : 1;
  prm.seed = seed;
  prm.lists = lists;
  prm.counts = counts;
  prm.err = err;
  prm.chunk_max = chunk_max;
  prm.chunk_stride = static_cast<int>(dense_chunk_stride(pl));
  prm.B = B;
  prm.N = N;
  prm.n_qsg = pl.n_qsg;
  prm.n_splits = pl.n_splits;
  prm.tile_stride = stride;
  prm.tile_offset = 0;
  prm.pass_tiles = (pl.tiles + stride - 1) / stride;
  prm.k = k;
  prm.cap = pl.cap;
  const int n_tasks = pl.n_qsg * pl.n_splits;
  cudaError_t e = cudaSuccess;
  const int kb = row_bytes / 128;
  const int epl = dense_epl(pl.cap);
  bool handled = false;
  if (pl.two_sm) {
    const int n_pairs = std::min(n_tasks, max_pairs());
#define RB_DISPATCH2F(ELEM, KB, NG, ST, F)                                                  \
  if (!handled && elem == ELEM && kb == KB && pl.ng == NG && filtered == F) {                \
    e = launch_2sm_variant<ELEM, KB, NG, ST, F>(mode, epl, prm, n_pairs, stream);            \
    handled = true;                                                                          \
  }
#define RB_DISPATCH2(ELEM, KB, NG, ST) RB_DISPATCH2F(ELEM, KB, NG, ST, false)
    RB_DISPATCH2(0, 1, 1, 12)
    RB_DISPATCH2(0, 1, 2, 12)
    RB_DISPATCH2(0, 2, 1, 8)
    RB_DISPATCH2(0, 2, 2, 8)
    RB_DISPATCH2(0, 4, 1, 4)
    RB_DISPATCH2(1, 1, 1, 12)
    RB_DISPATCH2(1, 1, 2, 12)
    RB_DISPATCH2(1, 2, 1, 8)
    RB_DISPATCH2(1, 2, 2, 8)
    RB_DISPATCH2(1, 4, 1, 4)
    RB_DISPATCH2(2, 1, 1, 12)
    RB_DISPATCH2(2, 1, 2, 12)
    RB_DISPATCH2(2, 2, 1, 8)
    RB_DISPATCH2(2, 2, 2, 8)
    RB_DISPATCH2(2, 4, 1, 4)
    // attribute-filtered variants (fp16 / bf16, rows of up to 256 bytes)
    RB_DISPATCH2F(0, 1, 1, 12, true)
    RB_DISPATCH2F(0, 1, 2, 12, true)
    RB_DISPATCH2F(0, 2, 1, 8, true)
    RB_DISPATCH2F(0, 2, 2, 8, true)
    RB_DISPATCH2F(1, 1, 1, 12, true)
    RB_DISPATCH2F(1, 1, 2, 12, true)
    RB_DISPATCH2F(1, 2, 1, 8, true)
    RB_DISPATCH2F(1, 2, 2, 8, true)
#undef RB_DISPATCH2
#undef RB_DISPATCH2F
  } else {
    const int grid = std::min(n_tasks, num_sms());
#define RB_DISPATCHF(ELEM, KB, NG, ST, F)                                                   \
  if (!handled && elem == ELEM && kb == KB && pl.ng == NG && filtered == F) {                \
    e = launch_1sm_variant<ELEM, KB, NG, ST, F>(mode, epl, prm, grid, stream);               \
    handled = true;                                                                          \
  }
#define RB_DISPATCH(ELEM, KB, NG, ST) RB_DISPATCHF(ELEM, KB, NG, ST, false)
    RB_DISPATCH(0, 1, 1, 8)
    RB_DISPATCH(0, 2, 1, 4)
    RB_DISPATCH(0, 4, 1, 2)
    RB_DISPATCH(1, 1, 1, 8)
    RB_DISPATCH(1, 2, 1, 4)
    RB_DISPATCH(1, 4, 1, 2)
    RB_DISPATCH(2, 1, 1, 8)
    RB_DISPATCH(2, 2, 1, 4)
    RB_DISPATCH(2, 4, 1, 2)
    RB_DISPATCHF(0, 1, 1, 8, true)
    RB_DISPATCHF(0, 2, 1, 4, true)
    RB_DISPATCHF(1, 1, 1, 8, true)
    RB_DISPATCHF(1, 2, 1, 4, true)
#undef RB_DISPATCH
#undef RB_DISPATCHF
  }
  if (!handled) {
    set_last_error("dense scan: unsupported dtype / row width");
    return RB_ERR_UNSUPPORTED;
  }
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

}  // namespace rb
