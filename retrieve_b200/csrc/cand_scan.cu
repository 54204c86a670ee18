// Scoring + exact top-k over per-query candidate lists, and the full-scan
// 1-bit Hamming top-k.
//
//  * retrieve::fused_masked_knn_topk (ops/triton/fused_masked_knn_topk.py:60-310;
//    twin ops/reference/fused_masked_knn_topk.py:9-29): candidates
//    positive_indices[b, :counts[b]], score = fp32 dot(query[b], item[id])
//    (fp16 / fp32 inputs widened to fp32), top-k, ids mapped back through
//    positive_indices, non-finite winners -> -1, lanes past counts never read
//    (and ids outside [0, N) never scored).
//  * retrieve::oporp_1bit_match_topk_indirect (ops/triton/oporp_1bit_match_topk.py
//    :47-292; twin ops/reference/oporp_1bit_match_topk.py:27-41): same
//    candidates, score = 64 W - 2 sum_w popc(q[w] ^ x[w]) as fp32; min(k, P)
//    columns, no padding.
//  * retrieve::oporp_1bit_match_topk_full (twin :17-24): every item, ids are
//    rows, no sentinel.
//  * st::search's scorer (kind 2, ivf_search.cu): int8 query codes against int8
//    item codes, exact int32 dot; raw score fp32(dot), or fp16(dot / divisor) on
//    the fp16 path (silvertorch/ops/csrc/fused_kmean_ann.cpp:196-200); returns
//    candidate slots, not ids.
//
// Candidate paths: one warp per (query, candidate range) scans 32 candidates
// per step (lane = candidate) and appends the passing ones to its own list
// with a ballot; lists are compacted exactly (rb_select.cuh) and merged per
// query (merge.cu). Ties on score go to the lower candidate index (lane).
// Full scan: one thread per query (128 queries per CTA), items staged in
// shared memory, the query's Hamming distance to each item computed on CUDA
// cores (xor + popc), and the running threshold checked after half the words.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>

#include "rb_capi_internal.h"
#include "rb_common.cuh"
#include "rb_select.cuh"

namespace rb {

constexpr int kCandWarps = 4;
constexpr int kCandCap = 256;  // list capacity of a candidate-scan warp

struct CandParams {
  const void* query;     // [B, D] (dot) or [B, W] int64 (hamming)
  const void* items;     // [N, D] or [N, W] int64
  const int64_t* pos;    // [B, P]
  const int64_t* counts; // [B]
  int B, P, D, N;
  int k;
  uint2* lists;          // [B, n_lists, cap]
  int* list_counts;      // [B, n_lists]
  int n_lists;
  int divisor;           // kind 2: -1 (int32 raw) or the fp16 path's divisor (> 0)
};

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f<float>(float v) {
  return v;
}

// fp32 dot of the staged query with item row `id`, k in order.
template <typename XT>
__device__ __forceinline__ float dot_row(const float* __restrict__ sq, const XT* __restrict__ row, int D) {
  float acc = 0.f;
  if constexpr (sizeof(XT) == 2) {
    if ((D & 7) == 0 && (reinterpret_cast<uintptr_t>(row) & 15u) == 0) {
      for (int d = 0; d < D; d += 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(row + d);
        const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h[i]);
          acc = fmaf(sq[d + 2 * i], f.x, acc);
          acc = fmaf(sq[d + 2 * i + 1], f.y, acc);
        }
      }
      return acc;
    }
  } else {
    if ((D & 3) == 0 && (reinterpret_cast<uintptr_t>(row) & 15u) == 0) {
      for (int d = 0; d < D; d += 4) {
        const float4 v = *reinterpret_cast<const float4*>(row + d);
        acc = fmaf(sq[d], v.x, acc);
        acc = fmaf(sq[d + 1], v.y, acc);
        acc = fmaf(sq[d + 2], v.z, acc);
        acc = fmaf(sq[d + 3], v.w, acc);
      }
      return acc;
    }
  }
  for (int d = 0; d < D; ++d) acc = fmaf(sq[d], to_f(row[d]), acc);
  return acc;
}

// Exact int32 dot of the staged int8 query with an int8 item row: 16 codes per
// 16-byte load and four dp4a when both rows allow it, else one code at a time.
__device__ __forceinline__ int dot_i8(const int8_t* __restrict__ sq, const int8_t* __restrict__ row, int D) {
  int acc = 0;
  if ((D & 15) == 0 && ((reinterpret_cast<uintptr_t>(row) | reinterpret_cast<uintptr_t>(sq)) & 15u) == 0) {
    for (int d = 0; d < D; d += 16) {
      const int4 x = *reinterpret_cast<const int4*>(row + d);
      const int4 q = *reinterpret_cast<const int4*>(sq + d);
      acc = __dp4a(x.x, q.x, acc);
      acc = __dp4a(x.y, q.y, acc);
      acc = __dp4a(x.z, q.z, acc);
      acc = __dp4a(x.w, q.w, acc);
    }
    return acc;
  }
  for (int d = 0; d < D; ++d) acc += static_cast<int>(sq[d]) * static_cast<int>(row[d]);
  return acc;
}

__device__ __forceinline__ float hamming_score(const uint64_t* __restrict__ sq, const uint64_t* __restrict__ row,
                                               int W) {
  int h = 0;
  for (int w = 0; w < W; ++w) h += __popcll(sq[w] ^ row[w]);
  return static_cast<float>(64 * W - 2 * h);
}

// KIND 0: dot with query type QT and item type XT; KIND 1: hamming (int64 words);
// KIND 2: int8 codes (QT = XT = int8_t). CAP: list capacity (k <= CAP - 32).
template <int KIND, typename QT, typename XT, int CAP = kCandCap>
__global__ void __launch_bounds__(32 * kCandWarps) cand_scan_kernel(CandParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ uint32_t hist_all[kCandWarps][256];
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int list_idx = blockIdx.x * kCandWarps + warp;
  // stage the query (fp32 for dots, raw words for hamming)
  if constexpr (KIND == 0) {
    float* sq = reinterpret_cast<float*>(smem_raw);
    const QT* qrow = static_cast<const QT*>(p.query) + static_cast<size_t>(b) * p.D;
    for (int i = threadIdx.x; i < p.D; i += blockDim.x) sq[i] = to_f(qrow[i]);
  } else if constexpr (KIND == 1) {
    uint64_t* sq = reinterpret_cast<uint64_t*>(smem_raw);
    const uint64_t* qrow = static_cast<const uint64_t*>(p.query) + static_cast<size_t>(b) * p.D;
    for (int i = threadIdx.x; i < p.D; i += blockDim.x) sq[i] = qrow[i];
  } else {
    int8_t* sq = reinterpret_cast<int8_t*>(smem_raw);
    const int8_t* qrow = static_cast<const int8_t*>(p.query) + static_cast<size_t>(b) * p.D;
    for (int i = threadIdx.x; i < p.D; i += blockDim.x) sq[i] = qrow[i];
  }
  __syncthreads();
  int64_t cnt64 = p.counts[b];
  const int cnt = static_cast<int>(cnt64 < 0 ? 0 : (cnt64 > p.P ? p.P : cnt64));
  // this warp's share of [0, cnt), in whole 32-lane chunks
  const int chunks = (cnt + 31) / 32;
  const int c_lo = static_cast<int>((static_cast<int64_t>(list_idx) * chunks) / p.n_lists);
  const int c_hi = static_cast<int>((static_cast<int64_t>(list_idx + 1) * chunks) / p.n_lists);
  uint2* list = p.lists + (static_cast<size_t>(b) * p.n_lists + list_idx) * CAP;
  int count = 0;
  float thresh = -INFINITY;
  const int64_t* prow = p.pos + static_cast<size_t>(b) * p.P;
  for (int c = c_lo; c < c_hi; ++c) {
    const int i = c * 32 + lane;
    float s = __int_as_float(0x7fc00000);  // NaN: never passes
    const int64_t id = (i < cnt) ? prow[i] : -1;
    if (id >= 0 && id < p.N) {  // ids outside the table are never scored
      if constexpr (KIND == 0) {
        s = dot_row<XT>(reinterpret_cast<const float*>(smem_raw),
                        static_cast<const XT*>(p.items) + static_cast<size_t>(id) * p.D, p.D);
      } else if constexpr (KIND == 1) {
        s = hamming_score(reinterpret_cast<const uint64_t*>(smem_raw),
                          static_cast<const uint64_t*>(p.items) + static_cast<size_t>(id) * p.D, p.D);
      } else {
        const int dot = dot_i8(reinterpret_cast<const int8_t*>(smem_raw),
                               static_cast<const int8_t*>(p.items) + static_cast<size_t>(id) * p.D, p.D);
        s = static_cast<float>(dot);
        if (p.divisor != -1) s = __half2float(__float2half_rn(__fdiv_rn(s, static_cast<float>(p.divisor))));
      }
    }
    const bool pass = s >= thresh;
    const uint32_t bal = __ballot_sync(RB_FULL_MASK, pass);
    if (bal) {
      if (count > CAP - 32) {
        // lane 0 holds the list; all lanes keep identical copies of its state
        warp_compact_lists<CAP / 32>(list, count, thresh, lane == 0, p.k, hist_all[warp]);
        count = __shfl_sync(RB_FULL_MASK, count, 0);
        thresh = __shfl_sync(RB_FULL_MASK, thresh, 0);
      }
      const bool pass2 = s >= thresh;
      const uint32_t bal2 = __ballot_sync(RB_FULL_MASK, pass2);
      if (pass2) list[count + __popc(bal2 & lanemask_lt())] = make_uint2(__float_as_uint(s), static_cast<uint32_t>(i));
      count += __popc(bal2);
    }
  }
  if (count > p.k) {
    warp_compact_lists<CAP / 32>(list, count, thresh, lane == 0, p.k, hist_all[warp]);
    count = __shfl_sync(RB_FULL_MASK, count, 0);
  }
  if (lane == 0) p.list_counts[static_cast<size_t>(b) * p.n_lists + list_idx] = count;
}

// Maps merged lanes to item ids: id = pos[b, lane]; non-finite scores -> -1.
__global__ void map_lane_ids_kernel(int64_t* __restrict__ ids, const float* __restrict__ scores,
                                    const int64_t* __restrict__ pos, int B, int P, int k) {
  const size_t n = static_cast<size_t>(B) * k;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int64_t lane = ids[i];
    const size_t b = i / k;
    ids[i] = (lane >= 0 && isfinite(scores[i])) ? pos[b * P + lane] : -1;
  }
}

// ---------------------------------------------------------------------------
// Full-scan Hamming top-k: thread per query.
// ---------------------------------------------------------------------------
constexpr int kHamQ = 128;      // queries per CTA
constexpr int kHamTile = 128;   // items per shared-memory tile
constexpr int kHamMaxW = 16;    // up to 1024-bit codes

struct HamParams {
  const uint64_t* qbits;  // [B, W]
  const uint64_t* xbits;  // [N, W]
  int B, N, W, k;
  int n_qg, n_splits, cap;
  uint2* lists;           // [B, n_splits, cap]
  int* counts;            // [B, n_splits]
};

template <int W, int EPL>
__global__ void __launch_bounds__(kHamQ) hamming_scan_kernel(HamParams p) {
  __shared__ __align__(16) uint64_t tile[2][kHamTile * W];
  __shared__ uint32_t hist_all[kHamQ / 32][256];
  const int warp = threadIdx.x >> 5;
  const int n_tasks = p.n_qg * p.n_splits;
  for (int t = blockIdx.x; t < n_tasks; t += gridDim.x) {
    const int qg = t % p.n_qg, split = t / p.n_qg;
    const int q = qg * kHamQ + threadIdx.x;
    const bool valid_q = q < p.B;
    uint64_t qw[W];
#pragma unroll
    for (int w = 0; w < W; ++w) qw[w] = valid_q ? p.qbits[static_cast<size_t>(q) * W + w] : 0ull;
    const int n_tiles = (p.N + kHamTile - 1) / kHamTile;
    const int lo = static_cast<int>((static_cast<int64_t>(split) * n_tiles) / p.n_splits);
    const int hi = static_cast<int>((static_cast<int64_t>(split + 1) * n_tiles) / p.n_splits);
    uint2* list = p.lists + (static_cast<size_t>(valid_q ? q : 0) * p.n_splits + split) * p.cap;
    int count = 0;
    float thresh = -INFINITY;
    int hmax = 64 * W;  // pass iff hamming <= hmax (same as score >= thresh)
    for (int tt = lo; tt < hi; ++tt) {
      __syncthreads();
      const int64_t base = static_cast<int64_t>(tt) * kHamTile;
      const int64_t rem = static_cast<int64_t>(p.N) - base;
      const int n_here = rem < kHamTile ? static_cast<int>(rem) : kHamTile;
      uint64_t* tl = tile[tt & 1];
      for (int i = threadIdx.x; i < kHamTile * W; i += kHamQ)
        tl[i] = (i < n_here * W) ? p.xbits[base * W + i] : 0ull;
      __syncthreads();
      // room for a whole tile of appends
      const bool need = valid_q && (count > p.cap - kHamTile);
      if (__any_sync(RB_FULL_MASK, need)) {
        warp_compact_lists<EPL>(list, count, thresh, need, p.k, hist_all[warp]);
        if (thresh > -INFINITY) hmax = static_cast<int>(floorf((64.f * W - thresh) * 0.5f));
      }
      for (int c = 0; c < kHamTile; c += 32) {
        int hv[32];
        bool any = false;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const uint64_t* x = tl + (c + j) * W;
          int h = 0;
#pragma unroll
          for (int w = 0; w < W / 2; ++w) h += __popcll(qw[w] ^ x[w]);
          hv[j] = h;
          any |= h <= hmax;
        }
        if (!__any_sync(RB_FULL_MASK, valid_q && any)) continue;
        any = false;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const uint64_t* x = tl + (c + j) * W;
          int h = hv[j];
#pragma unroll
          for (int w = W / 2; w < W; ++w) h += __popcll(qw[w] ^ x[w]);
          hv[j] = h;
          any |= h <= hmax;
        }
        if (!__any_sync(RB_FULL_MASK, valid_q && any)) continue;
        if (valid_q) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (hv[j] <= hmax && c + j < n_here) {
              const float s = static_cast<float>(64 * W - 2 * hv[j]);
              list[count++] = make_uint2(__float_as_uint(s), static_cast<uint32_t>(base + c + j));
            }
          }
        }
      }
    }
    const bool need = valid_q && count > p.k;
    warp_compact_lists<EPL>(list, count, thresh, need, p.k, hist_all[warp]);
    if (valid_q) p.counts[static_cast<size_t>(q) * p.n_splits + split] = count;
  }
}

template <int EPL>
static void launch_hamming(int W, int grid, const HamParams& prm, cudaStream_t s) {
  switch (W) {
    case 2: hamming_scan_kernel<2, EPL><<<grid, kHamQ, 0, s>>>(prm); break;
    case 4: hamming_scan_kernel<4, EPL><<<grid, kHamQ, 0, s>>>(prm); break;
    case 6: hamming_scan_kernel<6, EPL><<<grid, kHamQ, 0, s>>>(prm); break;
    case 8: hamming_scan_kernel<8, EPL><<<grid, kHamQ, 0, s>>>(prm); break;
    case 10: hamming_scan_kernel<10, EPL><<<grid, kHamQ, 0, s>>>(prm); break;
    case 12: hamming_scan_kernel<12, EPL><<<grid, kHamQ, 0, s>>>(prm); break;
    case 14: hamming_scan_kernel<14, EPL><<<grid, kHamQ, 0, s>>>(prm); break;
    default: hamming_scan_kernel<16, EPL><<<grid, kHamQ, 0, s>>>(prm); break;
  }
}

static int check_launch() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

struct CandPlan {
  int ctas_per_query;
  int n_lists;
};

static CandPlan cand_plan(int B, int P) {
  // aim at >= 2 waves of 4-warp CTAs, and >= 16 candidate chunks per warp
  const int chunks = std::max(1, (P + 31) / 32);
  int per_q = std::max(1, (2 * 4 * num_sms() + B - 1) / std::max(B, 1));
  per_q = std::min(per_q, std::max(1, chunks / (16 * kCandWarps)));
  per_q = std::min(per_q, 256);
  return CandPlan{per_q, per_q * kCandWarps};
}

static size_t cand_ws_bytes(int B, int P) {
  const CandPlan pl = cand_plan(B, P);
  const size_t lists = align_up(static_cast<size_t>(B) * pl.n_lists * kCandCap * sizeof(uint2), 256) +
                       align_up(static_cast<size_t>(B) * pl.n_lists * sizeof(int), 256);
  // the Hamming candidate scan past 224 winners runs the counting select (W <= 16, k <= P)
  return std::max(lists, ham_select_ws_bytes(B, P, 16, P));
}

// The int8 scan's list capacity: 256 entries up to k = 224, 1280 (40 a lane) up to k = 1024.
constexpr int kCandCapLarge = 1280;
static int cand_i8_cap(int k) { return k <= kCandCap - 32 ? kCandCap : kCandCapLarge; }

size_t cand_i8_ws_bytes(int B, int P, int k) {
  const CandPlan pl = cand_plan(B, P);
  return align_up(static_cast<size_t>(B) * pl.n_lists * cand_i8_cap(k) * sizeof(uint2), 256) +
         align_up(static_cast<size_t>(B) * pl.n_lists * sizeof(int), 256);
}

int cand_i8_max_k() { return 1024; }

int cand_i8_topk(const int8_t* q_codes, const int8_t* items, int N, int D, const int64_t* pos, int P,
                 const int64_t* counts, int B, int k, int divisor, int64_t* out_slots, float* out_raw, void* workspace,
                 cudaStream_t s, uint2* out_pairs) {
  const CandPlan pl = cand_plan(B, P);
  const int cap = cand_i8_cap(k);
  uint2* lists = static_cast<uint2*>(workspace);
  int* lcounts = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) +
                                        align_up(static_cast<size_t>(B) * pl.n_lists * cap * sizeof(uint2), 256));
  CandParams prm{q_codes, items, pos, counts, B, P, D, N, k, lists, lcounts, pl.n_lists, divisor};
  const dim3 grid(pl.ctas_per_query, B);
  const size_t smem = align_up(static_cast<size_t>(D), 16);
  if (cap == kCandCap)
    cand_scan_kernel<2, int8_t, int8_t, kCandCap><<<grid, 32 * kCandWarps, smem, s>>>(prm);
  else
    cand_scan_kernel<2, int8_t, int8_t, kCandCapLarge><<<grid, 32 * kCandWarps, smem, s>>>(prm);
  const int rc = check_launch();
  if (rc != RB_OK) return rc;
  return merge_lists(lists, lcounts, B, pl.n_lists, cap, k, 0, out_slots, out_raw, out_pairs, s);
}

// Hamming full-scan plan
struct HamPlan {
  int n_qg, n_splits, cap;
};
static HamPlan ham_plan(int B, int N, int k) {
  HamPlan h;
  h.n_qg = (B + kHamQ - 1) / kHamQ;
  const int n_tiles = std::max(1, (N + kHamTile - 1) / kHamTile);
  h.n_splits = std::max(1, std::min(n_tiles, (4 * num_sms()) / h.n_qg));
  // k survivors + one tile of appends, multiple of 32: <= 512 entries (16 per
  // lane in the register compaction) up to k = 352, <= 1184 (40 per lane) above
  h.cap = ((k + kHamTile + 32) + 31) / 32 * 32;
  return h;
}
static size_t ham_ws_bytes(int B, int N, int k) {
  const HamPlan h = ham_plan(B, N, k);
  return align_up(static_cast<size_t>(B) * h.n_splits * h.cap * sizeof(uint2), 256) +
         align_up(static_cast<size_t>(B) * h.n_splits * sizeof(int), 256);
}

}  // namespace rb

using namespace rb;

extern "C" {

int rb_candidate_topk_workspace_size(int B, int P, size_t* bytes) {
  if (bytes == nullptr || B < 0 || P < 0) {
    set_last_error("candidate_topk_workspace_size: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  *bytes = cand_ws_bytes(B, P);
  return RB_OK;
}

// kind: 0 = dot product (query_dtype / item_dtype in {RB_F16, RB_F32}), 1 = hamming
// over int64 words (D = W). k_out = k (dot) or min(k, P) (hamming).
int rb_candidate_topk(int kind, const void* query, int query_dtype, const void* items, int item_dtype, int N, int D,
                      const int64_t* positive_indices, int P, const int64_t* counts, int B, int k,
                      int64_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes, void* stream) {
  if (B < 0 || P < 0 || D <= 0 || k < 1 || N < 0) {
    set_last_error("candidate_topk: bad sizes");
    return RB_ERR_INVALID_ARG;
  }
  if (kind == 0 && k > 1024) {
    set_last_error("candidate_topk: k > 1024 is not supported");
    return RB_ERR_UNSUPPORTED;
  }
  if (kind == 0 && ((query_dtype != RB_F16 && query_dtype != RB_F32) || (item_dtype != RB_F16 && item_dtype != RB_F32))) {
    set_last_error("candidate_topk: query and item_embs must be float16 or float32");
    return RB_ERR_TYPE;
  }
  if (kind == 0 && k > kCandCap - 32) {
    set_last_error("candidate_topk: k > 224 is not supported on the candidate path");
    return RB_ERR_UNSUPPORTED;
  }
  const int k_sel = (kind == 1) ? std::min(k, std::max(P, 0)) : k;
  if (B == 0 || k_sel == 0) return RB_OK;
  if (workspace == nullptr || workspace_bytes < cand_ws_bytes(B, P)) {
    set_last_error("candidate_topk: workspace too small");
    return RB_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (kind == 1 && k_sel > kCandCap - 32) {  // more winners than the lists hold: the counting select
    if (D > 16) {
      set_last_error("candidate_topk: the Hamming candidate scan takes at most 16 words");
      return RB_ERR_UNSUPPORTED;
    }
    return ham_select_topk(static_cast<const uint64_t*>(query), static_cast<const uint64_t*>(items), N, D,
                           positive_indices, P, counts, B, k_sel, out_ids, out_scores, workspace, workspace_bytes, s);
  }
  const CandPlan pl = cand_plan(B, P);
  uint2* lists = static_cast<uint2*>(workspace);
  int* lcounts = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) +
                                        align_up(static_cast<size_t>(B) * pl.n_lists * kCandCap * sizeof(uint2), 256));
  CandParams prm{query, items, positive_indices, counts, B, P, D, N, k_sel, lists, lcounts, pl.n_lists, 0};
  const dim3 grid(pl.ctas_per_query, B);
  const size_t smem = (kind == 0) ? static_cast<size_t>(D) * sizeof(float) : static_cast<size_t>(D) * 8;
  if (kind == 1)
    cand_scan_kernel<1, uint64_t, uint64_t><<<grid, 32 * kCandWarps, smem, s>>>(prm);
  else if (query_dtype == RB_F16 && item_dtype == RB_F16)
    cand_scan_kernel<0, __half, __half><<<grid, 32 * kCandWarps, smem, s>>>(prm);
  else if (query_dtype == RB_F16 && item_dtype == RB_F32)
    cand_scan_kernel<0, __half, float><<<grid, 32 * kCandWarps, smem, s>>>(prm);
  else if (query_dtype == RB_F32 && item_dtype == RB_F16)
    cand_scan_kernel<0, float, __half><<<grid, 32 * kCandWarps, smem, s>>>(prm);
  else
    cand_scan_kernel<0, float, float><<<grid, 32 * kCandWarps, smem, s>>>(prm);
  int rc = check_launch();
  if (rc != RB_OK) return rc;
  rc = merge_lists(lists, lcounts, B, pl.n_lists, kCandCap, k_sel, 0, out_ids, out_scores, nullptr, s);
  if (rc != RB_OK) return rc;
  const size_t n = static_cast<size_t>(B) * k_sel;
  map_lane_ids_kernel<<<static_cast<int>(std::min<size_t>((n + 255) / 256, 1024)), 256, 0, s>>>(
      out_ids, out_scores, positive_indices, B, P, k_sel);
  return check_launch();
}

int rb_hamming_topk_workspace_size(int B, int N, int W, int k, size_t* bytes) {
  if (bytes == nullptr || B < 0 || N < 0 || W <= 0 || k < 1) {
    set_last_error("hamming_topk_workspace_size: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  *bytes = (k > 1024 || (W & 1)) ? ham_select_ws_bytes(B, N, W, k) : ham_ws_bytes(B, N, k);
  return RB_OK;
}

int rb_hamming_topk(const int64_t* query_bits, const int64_t* item_bits, int B, int N, int W, int k,
                    int64_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes, void* stream) {
  if (B < 0 || N < 0 || W <= 0 || k < 1) {
    set_last_error("hamming_topk: bad sizes");
    return RB_ERR_INVALID_ARG;
  }
  if (W > kHamMaxW) {
    set_last_error("hamming_topk: at most 16 words");
    return RB_ERR_UNSUPPORTED;
  }
  if (B == 0) return RB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (N == 0) {
    fill_empty(out_ids, out_scores, static_cast<size_t>(B) * k, s);
    return check_launch();
  }
  if (k > 1024 || (W & 1)) {  // past the list kernel (k, or an odd word count): the counting select
    if (workspace == nullptr || workspace_bytes < ham_select_ws_bytes(B, N, W, k)) {
      set_last_error("hamming_topk: workspace too small");
      return RB_ERR_WORKSPACE;
    }
    return ham_select_topk(reinterpret_cast<const uint64_t*>(query_bits), reinterpret_cast<const uint64_t*>(item_bits),
                           N, W, nullptr, N, nullptr, B, k, out_ids, out_scores, workspace, workspace_bytes, s);
  }
  if (workspace == nullptr || workspace_bytes < ham_ws_bytes(B, N, k)) {
    set_last_error("hamming_topk: workspace too small");
    return RB_ERR_WORKSPACE;
  }
  const HamPlan h = ham_plan(B, N, k);
  uint2* lists = static_cast<uint2*>(workspace);
  int* lcounts = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) +
                                        align_up(static_cast<size_t>(B) * h.n_splits * h.cap * sizeof(uint2), 256));
  HamParams prm{reinterpret_cast<const uint64_t*>(query_bits), reinterpret_cast<const uint64_t*>(item_bits), B, N, W, k,
                h.n_qg, h.n_splits, h.cap, lists, lcounts};
  const int grid = std::min(h.n_qg * h.n_splits, 4 * num_sms());
  if (h.cap <= 512)
    launch_hamming<16>(W, grid, prm, s);
  else
    launch_hamming<40>(W, grid, prm, s);
  const int rc = check_launch();
  if (rc != RB_OK) return rc;
  return merge_lists(lists, lcounts, B, h.n_splits, h.cap, k, 0, out_ids, out_scores, nullptr, s);
}

}  // extern "C"
