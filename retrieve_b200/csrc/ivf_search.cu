// SilverTorch's IVF probe search: st::search and st::probe_prep
// (silvertorch/ops/csrc/fork_search.cpp:13-49; fork_search_cuda.cu:1256-1546).
//
// One rb_st_search call is five launches on the caller's stream:
//  1. quantize_int8_rows_kernel (quantize.cu): the query rows to int8 codes and
//     fp32 scales as the reference's prep computes them
//     (fork_search_cuda.cu:680-700).
//  2. probe_expand_kernel, one CTA per query row: the row's probed clusters to
//     the sorted-table positions it scores, in the reference scorer's slot
//     order: every probed cluster's warp-aligned prefix (32 * (len / 32)
//     positions) in probe order, then every cluster's remainder (len % 32) in
//     probe order (fused_kmean_ann_cuda.cu:100-110, 183-215). A position whose
//     bit is clear in the full-N filter mask, or that fails the exact clause
//     filter (fork_filters.cuh:15-41), becomes -1 and is never scored; the
//     mask is read high bit first, bit 63 - d % 64 of word d / 64
//     (bloom_index_util.cuh:138-180).
//  3. cand_scan_kernel<2> (cand_scan.cu): exact int32 dots of the int8 codes,
//     ranked on fp32(dot) or on fp16(dot / divisor); every |dot| <= 2^24 when
//     D <= 1024, so the fp32 value orders exactly as the int32 raw score.
//     Per-warp candidate lists, then
//  4. merge_lists_kernel (merge.cu): the exact top-k per row, ties to the lower
//     slot, the reference's tie order (fork_search_cuda.cu:1374-1480).
//  5. st_epilogue_kernel: id = sort_perm[position]; int32 path score =
//     (fp32(dot) * q_scale) * global_scale, fp16 path score =
//     raw * ((q_scale * divisor) * global_scale), each product rounded to fp32
//     (fork_search_cuda.cu:560-591); -1 / -inf past the candidates.
//
// Every global access is bounds-checked against the sizes passed in: a probe
// id outside [0, n_lists) scores as an empty cluster, cluster ranges are
// clipped to [0, N), and slots past the row width are dropped (the
// reference's CUDA scorer requires the probed total to fit the width and does
// not check it).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cstdint>

#include "rb_capi_internal.h"
#include "rb_common.cuh"
#include "rb_select.cuh"
#include "st_filters.cuh"

namespace rb {

constexpr int kExpandThreads = 256;
constexpr int kMaxProbes = 2048;  // per-probe table: 20 bytes a probe in shared memory
constexpr int kMaxSearchD = 1024;

// Block-wide inclusive scan of two int64 values (kExpandThreads threads).
__device__ __forceinline__ void block_scan2(int64_t (&part)[2][kExpandThreads], int64_t& a, int64_t& b) {
  const int tid = threadIdx.x;
  part[0][tid] = a;
  part[1][tid] = b;
  __syncthreads();
  for (int off = 1; off < kExpandThreads; off <<= 1) {
    int64_t x = 0, y = 0;
    if (tid >= off) {
      x = part[0][tid - off];
      y = part[1][tid - off];
    }
    __syncthreads();
    part[0][tid] += x;
    part[1][tid] += y;
    __syncthreads();
  }
  a = part[0][tid];
  b = part[1][tid];
}

__global__ void __launch_bounds__(kExpandThreads) probe_expand_kernel(
    const int64_t* __restrict__ probe_ids, int P, const int64_t* __restrict__ offsets,
    const int64_t* __restrict__ sizes, int64_t n_lists, int64_t N, FilterSet f, int width, int64_t pos_lo,
    int64_t pos_hi, int64_t* __restrict__ pos, int64_t* __restrict__ counts,
    const int64_t* __restrict__ pair_lengths = nullptr, PartialMask pm = PartialMask{nullptr, nullptr, nullptr, 0, 0}) {
  // per probe: start (int64), len, head slot, tail slot (int32, slots clipped to width)
  extern __shared__ __align__(16) uint8_t sm[];
  int64_t* p_start = reinterpret_cast<int64_t*>(sm);
  int* p_len = reinterpret_cast<int*>(sm + sizeof(int64_t) * P);
  int* p_head = p_len + P;
  int* p_tail = p_head + P;
  __shared__ int64_t part[2][kExpandThreads];

  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const int64_t* prow = probe_ids + static_cast<int64_t>(b) * P;
  const int per = (P + kExpandThreads - 1) / kExpandThreads;
  const int j0 = min(P, tid * per);
  const int j1 = min(P, j0 + per);
  int64_t head = 0, tail = 0;
  for (int j = j0; j < j1; ++j) {
    int64_t start, len;
    // cluster lengths from the cluster table, or given per (row, probe) (st::fused_kmean_ann)
    if (pair_lengths != nullptr)
      probe_range_len(offsets, n_lists, N, prow[j], pair_lengths[static_cast<int64_t>(b) * P + j], start, len);
    else
      probe_range(offsets, sizes, n_lists, N, prow[j], start, len);
    // A cluster longer than the row contributes at most the row. width is a
    // multiple of 32, so the clipped cluster is whole warps and every later
    // slot lands past the width, as it would unclipped.
    if (len > width) len = width;
    p_start[j] = start;
    p_len[j] = static_cast<int>(len);
    head += len / 32 * 32;
    tail += len % 32;
  }
  int64_t head_incl = head, tail_incl = tail;
  block_scan2(part, head_incl, tail_incl);
  const int64_t total_head = part[0][kExpandThreads - 1];
  const int64_t total_tail = part[1][kExpandThreads - 1];
  int64_t h = head_incl - head;               // first head slot of this thread's probes
  int64_t t = total_head + tail_incl - tail;  // first tail slot
  for (int j = j0; j < j1; ++j) {
    const int64_t len = p_len[j];
    p_head[j] = static_cast<int>(h < width ? h : width);
    p_tail[j] = static_cast<int>(t < width ? t : width);
    h += len / 32 * 32;
    t += len % 32;
  }
  __syncthreads();
  const int64_t total = total_head + total_tail;
  if (tid == 0) counts[b] = total < width ? total : width;

  const int warp = tid >> 5, lane = tid & 31;
  int64_t* out = pos + static_cast<int64_t>(b) * width;
  if (f.bloom.index != nullptr && pm.cumsum == nullptr) {
    // The bloom plan gives one 64-bit word per 64-doc column: each lane evaluates the plan on
    // one of 32 consecutive columns, and every position takes its bit from the lane that
    // holds its column's word (one evaluation per column instead of one per position).
    const int64_t plan = f.bloom.plan_index ? f.bloom.plan_index[b] : b;
    for (int j = warp; j < P; j += kExpandThreads / 32) {
      const int64_t start = p_start[j];
      const int len = p_len[j];
      if (len == 0) continue;
      const int full = len / 32 * 32;
      const int64_t hs = p_head[j], ts = p_tail[j];
      const int64_t c_last = (start + len - 1) >> 6;
      for (int64_t cb = start >> 6; cb <= c_last; cb += 32) {
        const uint64_t word = cb + lane <= c_last ? bloom_plan_word(f.bloom, plan, cb + lane) : 0ull;
        const int64_t lo = max(start, cb * 64), hi = min(start + len, (cb + 32) * 64);
        for (int64_t p0 = lo; p0 < hi; p0 += 32) {  // warp-uniform: every lane takes part in the shuffle
          const int64_t position = p0 + lane;
          const uint64_t w = __shfl_sync(RB_FULL_MASK, word, static_cast<int>(((position >> 6) - cb) & 31));
          if (position >= hi) continue;
          const int64_t i = position - start;
          const int64_t slot = i < full ? hs + i : ts + (i - full);
          if (slot >= width) continue;
          const bool keep = position >= pos_lo && position < pos_hi && ((w >> (63 - (position & 63))) & 1ull) &&
                            pos_passes<false>(f, b, position);
          out[slot] = keep ? position - pos_lo : -1;
        }
      }
    }
    return;
  }
  // slot <- position, the i-th doc of probe j's range
  auto emit = [&](int64_t slot, int64_t position, int j, int i) {
    if (slot >= width) return;
    // positions outside this table's window [pos_lo, pos_hi) keep their slot but are not scored;
    // the scorer reads the row position - pos_lo of its table
    const bool in = position >= pos_lo && position < pos_hi;
    const bool keep = in && pos_passes<true>(f, b, position) &&
                      (pm.cumsum == nullptr || partial_mask_pass(pm, b, j, i));
    out[slot] = keep ? position - pos_lo : -1;
  };
  for (int j = warp; j < P; j += kExpandThreads / 32) {
    const int64_t start = p_start[j];
    const int len = p_len[j];
    const int full = len / 32 * 32;
    const int64_t hs = p_head[j], ts = p_tail[j];
    for (int i = lane; i < full; i += 32) emit(hs + i, start + i, j, i);
    for (int i = lane; i < len - full; i += 32) emit(ts + i, start + full + i, j, full + i);
  }
}

// st::fused_kmean_ann's output (fused_kmean_ann_cuda.cu:2126-2262): per (row, slot) of the
// row's slot layout the raw score of the position there — the int32 dot, or
// fp16(fp32(dot) / divisor) — and the position as int32; empty, filtered and padding slots
// hold the dtype's lowest value (INT32_MIN, or -65504 = 0xfbff) and invalid_index_value.
// With a per-doc fp16 scale (per_embedding_scale, which takes the divisor's place) the raw
// score is fp16(fp32(fp16(dot)) / fp32(scale[p])): the CUDA scorer divides a Half by a Half
// (index_mm_helpers.cuh:49-53), the dot rounded to fp16 first.
template <bool HALF>
__global__ void raw_scores_kernel(const int8_t* __restrict__ items, int64_t N, int D, const int8_t* __restrict__ q,
                                  const int64_t* __restrict__ pos, const int64_t* __restrict__ counts, int width,
                                  int divisor, const __half* __restrict__ scale, int invalid,
                                  void* __restrict__ out_raw, int32_t* __restrict__ out_idx) {
  extern __shared__ __align__(16) uint8_t raw_sm[];
  int8_t* sq = reinterpret_cast<int8_t*>(raw_sm);
  const int64_t b = blockIdx.y;
  for (int d = threadIdx.x; d < D; d += blockDim.x) sq[d] = q[b * D + d];
  __syncthreads();
  const int64_t slot = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (slot >= width) return;
  const int64_t o = b * width + slot;
  const int64_t p = slot < counts[b] ? pos[o] : -1;
  if (p < 0 || p >= N) {
    if constexpr (HALF)
      reinterpret_cast<__half*>(out_raw)[o] = __ushort_as_half(0xfbffu);
    else
      reinterpret_cast<int32_t*>(out_raw)[o] = INT32_MIN;
    out_idx[o] = invalid;
    return;
  }
  const int8_t* row = items + p * D;
  int acc = 0;
  if ((D & 15) == 0 && (reinterpret_cast<uintptr_t>(row) & 15u) == 0) {
    for (int d = 0; d < D; d += 16) {
      const int4 x = *reinterpret_cast<const int4*>(row + d);
      const int4 y = *reinterpret_cast<const int4*>(sq + d);
      acc = __dp4a(x.x, y.x, acc);
      acc = __dp4a(x.y, y.y, acc);
      acc = __dp4a(x.z, y.z, acc);
      acc = __dp4a(x.w, y.w, acc);
    }
  } else {
    for (int d = 0; d < D; ++d) acc += static_cast<int>(row[d]) * static_cast<int>(sq[d]);
  }
  if constexpr (HALF) {
    const float num = scale ? __half2float(__float2half_rn(static_cast<float>(acc))) : static_cast<float>(acc);
    const float den = scale ? __half2float(scale[p]) : static_cast<float>(divisor);
    reinterpret_cast<__half*>(out_raw)[o] = __float2half_rn(__fdiv_rn(num, den));
  } else
    reinterpret_cast<int32_t*>(out_raw)[o] = acc;
  out_idx[o] = static_cast<int32_t>(p);
}

// st::fused_kmean_ann on float embeddings (fp32, fp16, bf16), the CUDA scorer's arithmetic
// (simple_index_mm.cuh:41-56, 96-151, 160-300): per doc one fused multiply-add chain per block
// of `unit` elements in element order — fp32 in one float, fp16 / bf16 in a packed pair (even
// elements in the low half, odd in the high), rounded at every step — the blocks added in
// order onto zero (a single block is taken as it is), the pair's halves added last. The raw
// score has the embeddings' type; divisor and per-doc scales do not apply.
template <typename T>
struct FloatDot;

template <>
struct FloatDot<float> {
  using Acc = float;
  __device__ static Acc zero() { return 0.0f; }
  __device__ static Acc block(const float* x, const float* q, int n) {
    float a = 0.0f;
    for (int i = 0; i < n; ++i) a = __fmaf_rn(x[i], q[i], a);
    return a;
  }
  __device__ static Acc add(Acc a, Acc b) { return __fadd_rn(a, b); }
  __device__ static float finish(Acc a) { return a; }
};

template <>
struct FloatDot<__half> {
  using Acc = __half2;
  __device__ static Acc zero() { return __float2half2_rn(0.0f); }
  __device__ static Acc block(const __half* x, const __half* q, int n) {
    __half2 a = zero();
    for (int i = 0; i < n; i += 2) a = __hfma2(__halves2half2(x[i], x[i + 1]), __halves2half2(q[i], q[i + 1]), a);
    return a;
  }
  __device__ static Acc add(Acc a, Acc b) { return __hadd2(a, b); }
  __device__ static __half finish(Acc a) { return __hadd(__low2half(a), __high2half(a)); }
};

template <>
struct FloatDot<__nv_bfloat16> {
  using Acc = __nv_bfloat162;
  __device__ static Acc zero() { return __float2bfloat162_rn(0.0f); }
  __device__ static Acc block(const __nv_bfloat16* x, const __nv_bfloat16* q, int n) {
    __nv_bfloat162 a = zero();
    for (int i = 0; i < n; i += 2)
      a = __hfma2(__halves2bfloat162(x[i], x[i + 1]), __halves2bfloat162(q[i], q[i + 1]), a);
    return a;
  }
  __device__ static Acc add(Acc a, Acc b) { return __hadd2(a, b); }
  __device__ static __nv_bfloat16 finish(Acc a) { return __hadd(__low2bfloat16(a), __high2bfloat16(a)); }
};

template <typename T>
__global__ void raw_scores_float_kernel(const T* __restrict__ items, int64_t N, int D, int unit,
                                        const T* __restrict__ q, const int64_t* __restrict__ pos,
                                        const int64_t* __restrict__ counts, int width, int invalid, T pad,
                                        T* __restrict__ out_raw, int32_t* __restrict__ out_idx) {
  extern __shared__ __align__(16) uint8_t fraw_sm[];
  T* sq = reinterpret_cast<T*>(fraw_sm);
  const int64_t b = blockIdx.y;
  for (int d = threadIdx.x; d < D; d += blockDim.x) sq[d] = q[b * D + d];
  __syncthreads();
  const int64_t slot = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (slot >= width) return;
  const int64_t o = b * width + slot;
  const int64_t p = slot < counts[b] ? pos[o] : -1;
  if (p < 0 || p >= N) {
    out_raw[o] = pad;
    out_idx[o] = invalid;
    return;
  }
  const T* row = items + p * D;
  using F = FloatDot<T>;
  typename F::Acc acc;
  if (D * static_cast<int>(sizeof(T)) <= 256) {  // one block, taken as it is
    acc = F::block(row, sq, D);
  } else {  // blocks added onto zero, even when one block is the whole row
    acc = F::zero();
    for (int b0 = 0; b0 < D; b0 += unit) acc = F::add(acc, F::block(row + b0, sq + b0, unit));
  }
  out_raw[o] = F::finish(acc);
  out_idx[o] = static_cast<int32_t>(p);
}

// Winners' slots and raw scores -> (ids, scores) [B, k]; columns past k_sel and
// slots outside [0, counts[b]) are -1 / -inf.
__global__ void st_epilogue_kernel(const int64_t* __restrict__ slots, const float* __restrict__ raw, int k_sel,
                                   const int64_t* __restrict__ pos, const int64_t* __restrict__ counts, int width,
                                   const int64_t* __restrict__ sort_perm, int64_t N, const float* __restrict__ q_scales,
                                   const float* __restrict__ global_scale, int divisor, int B, int k,
                                   int64_t* __restrict__ ids, float* __restrict__ scores) {
  const int64_t n = static_cast<int64_t>(B) * k;
  const float gs = *global_scale;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = i / k;
    const int j = static_cast<int>(i - b * k);
    int64_t id = -1;
    float score = -INFINITY;
    if (j < k_sel) {
      const int64_t slot = slots[b * k_sel + j];
      if (slot >= 0 && slot < counts[b] && slot < width) {
        const int64_t p = pos[b * width + slot];
        if (p >= 0 && p < N) {
          id = sort_perm[p];
          const float r = raw[b * k_sel + j];
          const float qs = q_scales[b];
          score = divisor == -1 ? __fmul_rn(__fmul_rn(r, qs), gs)
                                : __fmul_rn(r, __fmul_rn(__fmul_rn(qs, static_cast<float>(divisor)), gs));
        }
      }
    }
    ids[i] = id;
    scores[i] = score;
  }
}

// st::probe_prep's layout outputs, one thread per (row, probe): the probed
// cluster ids, lengths and offsets, and the warp count of each; then the
// per-row cumsum of warp-rounded lengths (one thread per row).
__global__ void probe_prep_gather_kernel(const int64_t* __restrict__ probe_ids, int B, int P,
                                         const int64_t* __restrict__ offsets, const int64_t* __restrict__ sizes,
                                         int64_t n_lists, int64_t* __restrict__ cluster_ids,
                                         int64_t* __restrict__ cluster_length, int64_t* __restrict__ cluster_offset,
                                         int32_t* __restrict__ warps) {
  const int64_t n = static_cast<int64_t>(B) * P;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = probe_ids[i];
    const bool ok = c >= 0 && c < n_lists;
    const int64_t len = ok ? sizes[c] : 0;
    cluster_ids[i] = c;
    cluster_length[i] = len;
    cluster_offset[i] = ok ? offsets[c] : 0;
    warps[i] = static_cast<int32_t>(len / 32);
  }
}

__global__ void probe_prep_row_cumsum_kernel(const int64_t* __restrict__ cluster_length, int B, int P,
                                             int32_t* __restrict__ rounded_cumsum) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int32_t acc = 0;
  for (int j = 0; j < P; ++j) {
    const int64_t len = cluster_length[static_cast<int64_t>(b) * P + j];
    acc += static_cast<int32_t>(len / 32 * 32);
    rounded_cumsum[static_cast<int64_t>(b) * P + j] = acc;
  }
}

// Global inclusive cumsums over all B * P (row, probe) pairs of len % 32 and of
// len / 32: one CTA, each thread a contiguous run.
__global__ void __launch_bounds__(kExpandThreads) probe_prep_global_cumsum_kernel(
    const int64_t* __restrict__ cluster_length, int64_t n, int32_t* __restrict__ rem_cumsum,
    int32_t* __restrict__ warp_cumsum) {
  __shared__ int64_t part[2][kExpandThreads];
  const int tid = threadIdx.x;
  const int64_t per = (n + kExpandThreads - 1) / kExpandThreads;
  const int64_t i0 = min(n, tid * per);
  const int64_t i1 = min(n, i0 + per);
  int64_t rem = 0, wrp = 0;
  for (int64_t i = i0; i < i1; ++i) {
    const int64_t len = cluster_length[i];
    rem += len % 32;
    wrp += len / 32;
  }
  int64_t rem_incl = rem, wrp_incl = wrp;
  block_scan2(part, rem_incl, wrp_incl);
  int64_t r = rem_incl - rem, w = wrp_incl - wrp;
  for (int64_t i = i0; i < i1; ++i) {
    const int64_t len = cluster_length[i];
    r += len % 32;
    w += len / 32;
    rem_cumsum[i] = static_cast<int32_t>(r);
    warp_cumsum[i] = static_cast<int32_t>(w);
  }
}

static int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

static int st_width(int max_tensor_size_per_row) { return (max_tensor_size_per_row + 31) / 32 * 32; }

// The filter of one call from the C-ABI struct: at most one of the mask, the exact
// clauses and the bloom plans (the reference's TORCH_CHECK, fork_search_cuda.cu:1282-1290;
// with plans and exact clauses together the caller passes the exact clauses only, as
// the bloom with its exact recheck returns the exact filter's result).
static int build_filters(const rb_st_filter* flt, int64_t N, FilterSet& fs) {
  fs = FilterSet{nullptr, 0, ExactArgs{nullptr, 0, 0, nullptr, nullptr, nullptr, 0},
                 BloomArgs{nullptr, 0, nullptr, 0, nullptr, 0, 0, nullptr, 0, 0}};
  if (flt == nullptr) return RB_OK;
  const int kinds = (flt->filtering_bit_mask != nullptr) + (flt->query_clause_attrs != nullptr) +
                    (flt->bloom_index != nullptr);
  if (kinds > 1) {
    set_last_error("st::search takes one filter: filtering_bit_mask, the exact clauses or the bloom plans");
    return RB_ERR_INVALID_ARG;
  }
  if (flt->filtering_bit_mask != nullptr) {
    if (flt->mask_words < 0) {
      set_last_error("st::search: bad filtering_bit_mask width");
      return RB_ERR_INVALID_ARG;
    }
    fs.mask = reinterpret_cast<const uint64_t*>(flt->filtering_bit_mask);
    fs.mask_words = flt->mask_words;
  }
  if (flt->query_clause_attrs != nullptr) {
    if (flt->item_clause_attrs == nullptr || flt->clause_slots == nullptr || flt->clause_is_reverse == nullptr ||
        flt->n_clauses < 0 || flt->attr_rows < 0 || flt->attr_docs < N) {
      set_last_error("st::search: the exact filter needs item_clause_attrs [R, >= N], clause_slots and "
                     "clause_is_reverse");
      return RB_ERR_INVALID_ARG;
    }
    fs.ex = ExactArgs{flt->item_clause_attrs, flt->attr_rows, flt->attr_docs, flt->clause_slots,
                      flt->clause_is_reverse, flt->query_clause_attrs, flt->n_clauses};
  }
  if (flt->bloom_index != nullptr) {
    if (flt->bundle_b_offsets == nullptr || flt->n_bundles < 1 || flt->plans == nullptr || flt->plan_count < 1 ||
        flt->plan_words < 8 * static_cast<int64_t>(flt->plan_count) || flt->bloom_words < 0 || flt->hash_k < 1 ||
        flt->bloom_k < 1) {
      set_last_error("st::search: the bloom filter needs bloom_index, bundle offsets, plans of plan_count slots, "
                     "bloom_k and hash_k");
      return RB_ERR_INVALID_ARG;
    }
    if (flt->bloom_k > kBloomMaxK || flt->max_stack_size > kBloomStack) {
      set_last_error("st::search: bloom_k > 10 or a plan stack deeper than 16 is not supported");
      return RB_ERR_UNSUPPORTED;
    }
    fs.bloom = BloomArgs{reinterpret_cast<const uint64_t*>(flt->bloom_index), flt->bloom_words,
                         flt->bundle_b_offsets, flt->n_bundles, flt->plans, flt->plan_words, flt->plan_count,
                         flt->query_plan_index, flt->bloom_k, flt->hash_k};
  }
  return RB_OK;
}

// Workspace: q codes [B, D] | q scales [B] | positions [B, width] | counts [B] |
// winner slots [B, k_sel] | winner raw scores [B, k_sel] | candidate lists.
struct StWs {
  size_t codes, scales, pos, counts, slots, raw, cand, total;
};

static StWs st_ws_layout(int B, int D, int width, int k_sel) {
  StWs w;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += align_up(bytes, 256);
    return at;
  };
  w.codes = take(static_cast<size_t>(B) * D);
  w.scales = take(static_cast<size_t>(B) * sizeof(float));
  w.pos = take(static_cast<size_t>(B) * width * sizeof(int64_t));
  w.counts = take(static_cast<size_t>(B) * sizeof(int64_t));
  w.slots = take(static_cast<size_t>(B) * k_sel * sizeof(int64_t));
  w.raw = take(static_cast<size_t>(B) * k_sel * sizeof(float));
  w.cand = take(cand_i8_ws_bytes(B, width, k_sel));
  w.total = off;
  return w;
}

static int st_check(int B, int D, int P, int64_t n_lists, int64_t N, int k, int max_tensor_size_per_row,
                    int divisor) {
  if (B < 0 || D <= 0 || P < 0 || n_lists < 0 || N < 0 || k < 1 || max_tensor_size_per_row < 0) {
    set_last_error("st::search: bad sizes");
    return RB_ERR_INVALID_ARG;
  }
  if (B > 65535) {
    set_last_error("st::search: more than 65535 query rows per call is not supported");
    return RB_ERR_UNSUPPORTED;
  }
  if (D > kMaxSearchD) {
    set_last_error("st::search: D > 1024 is not supported (the raw int32 dot must stay exact in fp32)");
    return RB_ERR_UNSUPPORTED;
  }
  if (P > kMaxProbes) {
    set_last_error("st::search: more than 2048 probes per row is not supported");
    return RB_ERR_UNSUPPORTED;
  }
  if (N > INT32_MAX || max_tensor_size_per_row > INT32_MAX - 31) {
    set_last_error("st::search: tables past 2^31 rows are not supported");
    return RB_ERR_UNSUPPORTED;
  }
  if (divisor != -1 && divisor <= 0) {
    set_last_error("st::search: divisor_for_int8 must be -1 or positive");
    return RB_ERR_INVALID_ARG;
  }
  const int k_sel = std::min(k, st_width(max_tensor_size_per_row));
  if (k_sel > cand_i8_max_k()) {
    set_last_error("st::search: min(k, padded width) > 1024 is not supported");
    return RB_ERR_UNSUPPORTED;
  }
  return RB_OK;
}

// ---------------------------------------------------------------------------
// Grouped scorer (rb_st_search_grouped): the same results as rb_st_search with
// each probed cluster read once per (cluster, group of probing rows) instead of
// once per probing row.
//
//  1. pair_count / cluster_scan / pair_scatter: the (row, probe) pairs grouped
//     by cluster (a counting sort; order inside a cluster is free, since every
//     pair owns its own candidate list); one task per cluster and group of at
//     most G pairs.
//  2. slot_starts: per pair, the row's first head slot and first tail slot of
//     that probe (the layout of probe_expand_kernel, cluster lengths clipped to
//     the width in the same way), and per row the total.
//  3. ivf_group_scan_kernel, one CTA per task: the pairs' query codes and then
//     128-row tiles of the cluster staged in shared memory; each warp takes
//     pairs and scores a whole tile for each (4 rows a lane, dp4a), appending
//     (raw score, slot) in ascending slot order to the pair's list, so ties keep
//     the lower slot exactly as in the row path. A compacted list holds k
//     candidates of its row at or above its k-th raw score; that score goes to
//     the row's bound (atomicMax), and every pair of the row skips what falls
//     under the bound from its next tile on (ties kept: the other pairs' slots
//     interleave with its own).
//  4. merge_lists over each row's P lists, then st_group_epilogue_kernel: slot
//     -> (probe, row in cluster) by binary search over the row's slot ends ->
//     position -> sort_perm, and the dequantization.
// ---------------------------------------------------------------------------
constexpr int kGroupThreads = 256;
constexpr int kGroupWarps = kGroupThreads / 32;
constexpr int kGroupTile = 128;  // cluster rows staged per step: 4 per lane
static_assert(kGroupTile <= 64 * 30, "a tile's bloom columns must fit the warp's lanes");
// candidate-list capacity per (row, probe): 256 entries up to k = 224, 1280 up to k = 1024
constexpr int kGroupCap = 256;
constexpr int kGroupCapLarge = 1280;
static int group_cap(int k) { return k <= kGroupCap - 32 ? kGroupCap : kGroupCapLarge; }
constexpr int kGroupMaxPairs = 64;

static int group_pairs_per_task(int D) {
  const int dp = (D + 15) / 16 * 16;
  return std::max(8, std::min(kGroupMaxPairs, 16384 / dp));
}

static size_t group_smem_bytes(int D) {
  const size_t dp = static_cast<size_t>(D + 15) / 16 * 16;
  return static_cast<size_t>(group_pairs_per_task(D)) * dp + kGroupTile * (dp + 16);
}

__global__ void pair_count_kernel(const int64_t* __restrict__ probe, int64_t n_pairs, int64_t n_lists,
                                  int* __restrict__ cnt) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_pairs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = probe[i];
    if (c >= 0 && c < n_lists) atomicAdd(&cnt[c], 1);
  }
}

// Exclusive prefix sums over clusters of the pair counts (cpo) and of the task
// counts ceil(cnt / G) (ctask), each with the total at index n_lists. One CTA.
__global__ void __launch_bounds__(kExpandThreads) cluster_scan_kernel(const int* __restrict__ cnt, int64_t n_lists,
                                                                      int G, int64_t* __restrict__ cpo,
                                                                      int64_t* __restrict__ ctask) {
  __shared__ int64_t part[2][kExpandThreads];
  const int tid = threadIdx.x;
  const int64_t per = (n_lists + kExpandThreads - 1) / kExpandThreads;
  const int64_t i0 = min(n_lists, tid * per);
  const int64_t i1 = min(n_lists, i0 + per);
  int64_t pairs = 0, tasks = 0;
  for (int64_t i = i0; i < i1; ++i) {
    pairs += cnt[i];
    tasks += (cnt[i] + G - 1) / G;
  }
  int64_t pairs_incl = pairs, tasks_incl = tasks;
  block_scan2(part, pairs_incl, tasks_incl);
  int64_t p = pairs_incl - pairs, t = tasks_incl - tasks;
  for (int64_t i = i0; i < i1; ++i) {
    cpo[i] = p;
    ctask[i] = t;
    p += cnt[i];
    t += (cnt[i] + G - 1) / G;
  }
  if (tid == kExpandThreads - 1) {
    cpo[n_lists] = pairs_incl;
    ctask[n_lists] = tasks_incl;
  }
}

__global__ void pair_scatter_kernel(const int64_t* __restrict__ probe, int64_t n_pairs, int64_t n_lists,
                                    const int64_t* __restrict__ cpo, int* __restrict__ fill,
                                    int32_t* __restrict__ pairs) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_pairs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = probe[i];
    if (c >= 0 && c < n_lists) pairs[cpo[c] + atomicAdd(&fill[c], 1)] = static_cast<int32_t>(i);
  }
}

// Per pair (row b, probe j): the row's first head and first tail slot of probe j;
// per row the slot total (before the width cut). One thread per row.
__global__ void slot_starts_kernel(const int64_t* __restrict__ probe, int B, int P, const int64_t* __restrict__ offsets,
                                   const int64_t* __restrict__ sizes, int64_t n_lists, int64_t N, int width,
                                   int64_t* __restrict__ head, int64_t* __restrict__ tail,
                                   int64_t* __restrict__ row_total) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int64_t o = static_cast<int64_t>(b) * P;
  row_total[b] = row_slot_starts(probe + o, P, offsets, sizes, n_lists, N, width, head + o, tail + o);
}

struct GroupArgs {
  const int8_t* items;  // [N, D], cluster-sorted
  int64_t N;
  int D;
  const int8_t* q_codes;  // [B, D]
  const int64_t* probe;   // [B, P]
  int P;
  const int64_t* offsets;
  const int64_t* sizes;
  int64_t n_lists;
  const int32_t* pairs;  // pair ids b * P + j, grouped by cluster
  const int64_t* cpo;    // [n_lists + 1]
  const int64_t* ctask;  // [n_lists + 1]
  const int64_t* head;   // [B * P]
  const int64_t* tail;   // [B * P]
  int width;
  int G;
  int k;
  int divisor;
  FilterSet f;
  uint2* lists;      // [B * P, CAP]
  int* list_counts;  // [B * P]
  uint32_t* row_bound;  // [B] f2ord of a lower bound on the row's k-th raw score (0: none yet)
};

template <int CAP, bool BLOOM>
__global__ void __launch_bounds__(kGroupThreads) ivf_group_scan_kernel(GroupArgs a) {
  extern __shared__ __align__(16) uint8_t gsm[];
  __shared__ uint32_t hist[kGroupWarps][256];
  __shared__ int s_pair[kGroupMaxPairs];
  __shared__ int s_count[kGroupMaxPairs];
  __shared__ float s_thresh[kGroupMaxPairs];

  const int64_t task = blockIdx.x;
  if (task >= a.ctask[a.n_lists]) return;  // the grid is an upper bound on the tasks
  // the cluster: the largest c with ctask[c] <= task (ctask[0] = 0, non-decreasing)
  int64_t lo = 0, hi = a.n_lists;
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (a.ctask[mid] <= task) lo = mid; else hi = mid;
  }
  const int64_t c = lo;
  const int64_t p0 = a.cpo[c] + (task - a.ctask[c]) * a.G;
  const int64_t p1 = min(p0 + a.G, a.cpo[c + 1]);
  const int m = static_cast<int>(p1 - p0);
  int64_t start, len, full;
  clipped_probe(a.offsets, a.sizes, a.n_lists, a.N, c, a.width, start, len, full);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int dp = (a.D + 15) & ~15;  // query row stride in shared memory
  const int rs = dp + 16;           // tile row stride: 8 lanes' 16-byte loads hit distinct banks
  int8_t* sq = reinterpret_cast<int8_t*>(gsm);
  int8_t* sx = sq + static_cast<size_t>(a.G) * dp;
  for (int g = tid; g < m; g += kGroupThreads) {
    s_pair[g] = a.pairs[p0 + g];
    s_count[g] = 0;
    s_thresh[g] = -INFINITY;
  }
  __syncthreads();
  for (int idx = tid; idx < m * dp; idx += kGroupThreads) {
    const int g = idx / dp, d = idx - g * dp;
    const int64_t b = s_pair[g] / a.P;
    sq[g * dp + d] = d < a.D ? a.q_codes[b * a.D + d] : static_cast<int8_t>(0);
  }
  const bool vec = (a.D & 15) == 0 && (reinterpret_cast<uintptr_t>(a.items) & 15u) == 0;
  for (int64_t t0 = 0; t0 < len; t0 += kGroupTile) {
    const int rows = static_cast<int>(min(static_cast<int64_t>(kGroupTile), len - t0));
    __syncthreads();  // the previous tile has been scored (and the query codes are staged)
    if (vec) {
      const int chunks = a.D / 16;
      for (int idx = tid; idx < kGroupTile * chunks; idx += kGroupThreads) {
        const int r = idx / chunks, ch = idx - r * chunks;
        int4 v = make_int4(0, 0, 0, 0);
        if (r < rows) v = *reinterpret_cast<const int4*>(a.items + (start + t0 + r) * a.D + ch * 16);
        *reinterpret_cast<int4*>(sx + r * rs + ch * 16) = v;
      }
    } else {
      for (int idx = tid; idx < kGroupTile * dp; idx += kGroupThreads) {
        const int r = idx / dp, d = idx - r * dp;
        sx[r * rs + d] = (r < rows && d < a.D) ? a.items[(start + t0 + r) * a.D + d] : static_cast<int8_t>(0);
      }
    }
    __syncthreads();
    for (int g = warp; g < m; g += kGroupWarps) {
      const int pr = s_pair[g];
      const int64_t b = pr / a.P;
      int count = s_count[g];
      // the row's bound: the k-th score of some compacted list of the row (another pair's rows
      // may have lower slots, so ties stay: the test is >=)
      float thresh = fmaxf(s_thresh[g], ord2f(__ldcg(a.row_bound + b)));
      uint2* list = a.lists + static_cast<int64_t>(pr) * CAP;
      const int64_t hs = a.head[pr], ts = a.tail[pr];
      const int4* q = reinterpret_cast<const int4*>(sq + g * dp);
      // bloom: the tile's rows span at most 3 64-doc columns; lanes 0..2 evaluate the row's plan
      // on them once, and each position takes its bit by shuffle
      uint64_t cword = 0;
      const int64_t cb = (start + t0) >> 6;
      if constexpr (BLOOM) {
        const int64_t c_last = (start + t0 + rows - 1) >> 6;
        const int64_t plan = a.f.bloom.plan_index ? a.f.bloom.plan_index[b] : b;
        if (cb + lane <= c_last) cword = bloom_plan_word(a.f.bloom, plan, cb + lane);
      }
#pragma unroll 1
      for (int r = 0; r < kGroupTile / 32; ++r) {
        const int li = r * 32 + lane;
        const int64_t i = t0 + li;  // row within the cluster
        const int64_t position = start + i;
        bool bit = true;
        if constexpr (BLOOM) {
          const uint64_t w = __shfl_sync(RB_FULL_MASK, cword, static_cast<int>(((position >> 6) - cb) & 31));
          bit = (w >> (63 - (position & 63))) & 1ull;
        }
        float s = __int_as_float(0x7fc00000);  // NaN: never passes
        uint32_t slot32 = 0;
        if (li < rows) {
          const int64_t slot = i < full ? hs + i : ts + (i - full);
          const bool ok = slot < a.width && bit && pos_passes<false>(a.f, b, position);
          if (ok) {
            const int4* x = reinterpret_cast<const int4*>(sx + li * rs);
            int acc = 0;
            for (int ch = 0; ch < dp / 16; ++ch) {
              const int4 xv = x[ch], qv = q[ch];
              acc = __dp4a(xv.x, qv.x, acc);
              acc = __dp4a(xv.y, qv.y, acc);
              acc = __dp4a(xv.z, qv.z, acc);
              acc = __dp4a(xv.w, qv.w, acc);
            }
            s = static_cast<float>(acc);
            if (a.divisor != -1) s = __half2float(__float2half_rn(__fdiv_rn(s, static_cast<float>(a.divisor))));
            slot32 = static_cast<uint32_t>(slot);
          }
        }
        const bool pass = s >= thresh;
        if (__ballot_sync(RB_FULL_MASK, pass)) {
          if (count > CAP - 32) {
            warp_compact_lists<CAP / 32>(list, count, thresh, lane == 0, a.k, hist[warp]);
            count = __shfl_sync(RB_FULL_MASK, count, 0);
            thresh = __shfl_sync(RB_FULL_MASK, thresh, 0);
            // the list now holds k candidates of the row at or above one step below thresh
            if (lane == 0) atomicMax(a.row_bound + b, f2ord(thresh) - 1u);
          }
          const bool pass2 = s >= thresh;
          const uint32_t bal2 = __ballot_sync(RB_FULL_MASK, pass2);
          if (pass2) list[count + __popc(bal2 & lanemask_lt())] = make_uint2(__float_as_uint(s), slot32);
          count += __popc(bal2);
        }
      }
      __syncwarp();
      if (lane == 0) {
        s_count[g] = count;
        s_thresh[g] = thresh;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  for (int g = warp; g < m; g += kGroupWarps) {
    const int pr = s_pair[g];
    int count = s_count[g];
    float thresh = s_thresh[g];
    if (count > a.k) {
      warp_compact_lists<CAP / 32>(a.lists + static_cast<int64_t>(pr) * CAP, count, thresh, lane == 0,
                                         a.k, hist[warp]);
      count = __shfl_sync(RB_FULL_MASK, count, 0);
      thresh = __shfl_sync(RB_FULL_MASK, thresh, 0);
      if (lane == 0) atomicMax(a.row_bound + pr / a.P, f2ord(thresh) - 1u);
    }
    if (lane == 0) a.list_counts[pr] = count;
  }
}

// Winners (slot, raw) -> (ids, scores): the slot's probe is the first j whose
// head (or tail) range ends past the slot; binary search over the row's starts.
__global__ void st_group_epilogue_kernel(const int64_t* __restrict__ slots, const float* __restrict__ raw, int k_sel,
                                         const int64_t* __restrict__ probe, int P, const int64_t* __restrict__ offsets,
                                         const int64_t* __restrict__ sizes, int64_t n_lists,
                                         const int64_t* __restrict__ head, const int64_t* __restrict__ tail,
                                         const int64_t* __restrict__ row_total, int width,
                                         const int64_t* __restrict__ sort_perm, int64_t N,
                                         const float* __restrict__ q_scales, const float* __restrict__ global_scale,
                                         int divisor, int B, int k, int64_t* __restrict__ ids,
                                         float* __restrict__ scores) {
  const int64_t n = static_cast<int64_t>(B) * k;
  const float gs = *global_scale;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = i / k;
    const int jo = static_cast<int>(i - b * k);
    int64_t id = -1;
    float score = -INFINITY;
    if (jo < k_sel && P > 0) {
      const int64_t slot = slots[b * k_sel + jo];
      const int64_t* hrow = head + b * P;
      const int64_t* trow = tail + b * P;
      if (slot >= 0 && slot < width && slot < row_total[b]) {
        bool in_head;
        const int lo = slot_to_probe(hrow, trow, row_total[b], P, slot, in_head);
        int64_t start, len, full;
        clipped_probe(offsets, sizes, n_lists, N, probe[b * P + lo], width, start, len, full);
        const int64_t in_cluster = in_head ? slot - hrow[lo] : full + (slot - trow[lo]);  // row in the cluster
        const int64_t p = start + in_cluster;
        if (in_cluster >= 0 && in_cluster < len && p >= 0 && p < N) {
          id = sort_perm[p];
          const float r = raw[b * k_sel + jo];
          const float qs = q_scales[b];
          score = divisor == -1 ? __fmul_rn(__fmul_rn(r, qs), gs)
                                : __fmul_rn(r, __fmul_rn(__fmul_rn(qs, static_cast<float>(divisor)), gs));
        }
      }
    }
    ids[i] = id;
    scores[i] = score;
  }
}

}  // namespace rb

using namespace rb;

extern "C" {

int rb_st_search_workspace_size(int B, int D, int P, int k, int max_tensor_size_per_row, size_t* bytes) {
  if (bytes == nullptr || B < 0 || D <= 0 || P < 0 || k < 1 || max_tensor_size_per_row < 0 ||
      max_tensor_size_per_row > INT32_MAX - 31) {
    set_last_error("st_search_workspace_size: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  const int width = st_width(max_tensor_size_per_row);
  *bytes = st_ws_layout(B, D, width, std::min(k, width)).total;
  return RB_OK;
}

}  // extern "C"

// The row path over the positions [pos_lo, pos_hi) of a table of n_total positions (the
// whole table: 0, n_total); item_codes holds the window's rows. With out_pairs the
// winners are written as (raw score bits, slot) pairs and nothing else; otherwise the
// epilogue writes ids (sort_perm indexed by position) and scores.
static int st_row_search(const float* query, int B, int D, const int64_t* probe_ids, int P,
                         const int64_t* cluster_offsets, const int64_t* cluster_sizes, int64_t n_lists,
                         int64_t n_total, int64_t pos_lo, int64_t pos_hi, const int8_t* item_codes,
                         const int64_t* sort_perm, const float* global_scale, int k, int max_tensor_size_per_row,
                         int divisor_for_int8, const rb_st_filter* filter, int64_t* out_ids, float* out_scores,
                         uint64_t* out_pairs, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = st_check(B, D, P, n_lists, n_total, k, max_tensor_size_per_row, divisor_for_int8);
  if (rc != RB_OK) return rc;
  if (pos_lo < 0 || pos_hi < pos_lo || pos_hi > n_total) {
    set_last_error("st::search: the position window must lie in [0, N]");
    return RB_ERR_INVALID_ARG;
  }
  FilterSet fs;
  rc = build_filters(filter, n_total, fs);
  if (rc != RB_OK) return rc;
  if (B == 0) return RB_OK;
  const int width = st_width(max_tensor_size_per_row);
  const int k_sel = std::min(k, width);
  const StWs lay = st_ws_layout(B, D, width, k_sel);
  if (workspace == nullptr || workspace_bytes < lay.total) {
    set_last_error("st::search: workspace too small");
    return RB_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int8_t* q_codes = reinterpret_cast<int8_t*>(ws + lay.codes);
  float* q_scales = reinterpret_cast<float*>(ws + lay.scales);
  int64_t* pos = reinterpret_cast<int64_t*>(ws + lay.pos);
  int64_t* counts = reinterpret_cast<int64_t*>(ws + lay.counts);
  int64_t* slots = reinterpret_cast<int64_t*>(ws + lay.slots);
  float* raw = reinterpret_cast<float*>(ws + lay.raw);

  rc = rb_quantize_int8(query, B, D, q_codes, q_scales, stream);
  if (rc != RB_OK) return rc;
  if (width == 0) {
    // nothing can be probed: every row is all -1 / -inf
    if (out_pairs != nullptr)
      fill_empty_pairs(reinterpret_cast<uint2*>(out_pairs), static_cast<size_t>(B) * k_sel, s);
    else
      fill_empty(out_ids, out_scores, static_cast<size_t>(B) * k, s);
    return launch_status();
  }
  const size_t smem = static_cast<size_t>(P) * (sizeof(int64_t) + 3 * sizeof(int));
  probe_expand_kernel<<<B, kExpandThreads, smem, s>>>(probe_ids, P, cluster_offsets, cluster_sizes, n_lists, n_total,
                                                      fs, width, pos_lo, pos_hi, pos, counts);
  rc = launch_status();
  if (rc != RB_OK) return rc;
  ProfileEvents& pe = profile_events();
  if (pe.start) record_profile_event(pe.start, s);
  rc = cand_i8_topk(q_codes, item_codes, static_cast<int>(pos_hi - pos_lo), D, pos, width, counts, B, k_sel,
                    divisor_for_int8, slots, raw, ws + lay.cand, s, reinterpret_cast<uint2*>(out_pairs));
  if (rc != RB_OK) return rc;
  if (pe.stop) record_profile_event(pe.stop, s);
  if (out_pairs != nullptr) return rc;
  const int64_t n = static_cast<int64_t>(B) * k;
  const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, 4096));
  st_epilogue_kernel<<<grid, 256, 0, s>>>(slots, raw, k_sel, pos, counts, width, sort_perm, n_total, q_scales,
                                          global_scale, divisor_for_int8, B, k, out_ids, out_scores);
  return launch_status();
}

namespace rb {

// The tensor-core form of the grouped scan (ivf_tc.cu): int8 rows of 128, 256 or
// 512 bytes, no bloom plans (lists of ivf_tc_cap entries).
bool ivf_tc_supported(int D, int k_sel, bool bloom);
int ivf_tc_cap(int k_sel);
size_t ivf_tc_ws_bytes(int64_t n_pairs, int64_t n_lists, int D);
int ivf_tc_scan(const int8_t* q_codes, int B, int D, int P, const int8_t* item_codes, int64_t N,
                const int64_t* offsets, const int64_t* sizes, int64_t n_lists, const int32_t* pairs,
                const int64_t* cpo, const int64_t* ctask, const int64_t* head, const int64_t* tail, int width,
                int k_sel, int divisor, const FilterSet& fs, uint2* lists, int* list_counts, uint32_t* row_bound,
                int* err, void* ws, cudaStream_t s);

// The SIMT grouped scan (ivf_group_scan_kernel) over the tasks of G pairs.
static int group_scan(const int8_t* item_codes, int64_t N, int D, const int8_t* q_codes, const int64_t* probe_ids,
                      int P, const int64_t* cluster_offsets, const int64_t* cluster_sizes, int64_t n_lists,
                      const int32_t* pairs, const int64_t* cpo, const int64_t* ctask, const int64_t* head,
                      const int64_t* tail, int width, int G, int k_sel, int divisor_for_int8, const FilterSet& fs,
                      uint2* lists, int* lcounts, uint32_t* row_bound, int64_t n_pairs, cudaStream_t s) {
  int rc = RB_OK;
  const size_t smem = group_smem_bytes(D);
  // the limit is a per-device setting of the function: raised once on each device used
  static std::atomic<uint64_t> smem_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const bool known = dev >= 0 && dev < 64;
  if (!known || !((smem_set.load() >> dev) & 1u)) {
    // the largest tile (D = 1024) needs about 150 KB of the 227 KB a block may opt into
    const int most = static_cast<int>(group_smem_bytes(kMaxSearchD));
    const auto attr = cudaFuncAttributeMaxDynamicSharedMemorySize;
    if (cudaFuncSetAttribute(ivf_group_scan_kernel<kGroupCap, false>, attr, most) != cudaSuccess ||
        cudaFuncSetAttribute(ivf_group_scan_kernel<kGroupCap, true>, attr, most) != cudaSuccess ||
        cudaFuncSetAttribute(ivf_group_scan_kernel<kGroupCapLarge, false>, attr, most) != cudaSuccess ||
        cudaFuncSetAttribute(ivf_group_scan_kernel<kGroupCapLarge, true>, attr, most) != cudaSuccess) {
      set_last_error("st::search: cannot raise the grouped scan's shared memory limit");
      return RB_ERR_CUDA;
    }
    if (known) smem_set.fetch_or(uint64_t{1} << dev);
  }
  const int64_t max_tasks = (n_pairs + G - 1) / G + std::min<int64_t>(n_lists, n_pairs);
  GroupArgs ga{item_codes, N, D, q_codes, probe_ids, P, cluster_offsets, cluster_sizes, n_lists, pairs, cpo, ctask,
               head, tail, width, G, k_sel, divisor_for_int8, fs, lists, lcounts, row_bound};
  const unsigned grid_tasks = static_cast<unsigned>(max_tasks);
  const bool bloom = fs.bloom.index != nullptr;
  ProfileEvents& pe = profile_events();
  if (pe.start) record_profile_event(pe.start, s);
  if (group_cap(k_sel) == kGroupCap) {
    if (bloom)
      ivf_group_scan_kernel<kGroupCap, true><<<grid_tasks, kGroupThreads, smem, s>>>(ga);
    else
      ivf_group_scan_kernel<kGroupCap, false><<<grid_tasks, kGroupThreads, smem, s>>>(ga);
  } else {
    if (bloom)
      ivf_group_scan_kernel<kGroupCapLarge, true><<<grid_tasks, kGroupThreads, smem, s>>>(ga);
    else
      ivf_group_scan_kernel<kGroupCapLarge, false><<<grid_tasks, kGroupThreads, smem, s>>>(ga);
  }
  rc = launch_status();
  if (rc != RB_OK) return rc;
  if (pe.stop) record_profile_event(pe.stop, s);
  return RB_OK;
}

}  // namespace rb

extern "C" {

int rb_st_search(const float* query, int B, int D, const int64_t* probe_ids, int P, const int64_t* cluster_offsets,
                 const int64_t* cluster_sizes, int64_t n_lists, const int8_t* item_codes, int64_t N,
                 const int64_t* sort_perm, const float* global_scale, int k, int max_tensor_size_per_row,
                 int divisor_for_int8, const rb_st_filter* filter, int64_t* out_ids, float* out_scores,
                 void* workspace, size_t workspace_bytes, void* stream) {
  return st_row_search(query, B, D, probe_ids, P, cluster_offsets, cluster_sizes, n_lists, N, 0, N, item_codes,
                       sort_perm, global_scale, k, max_tensor_size_per_row, divisor_for_int8, filter, out_ids,
                       out_scores, nullptr, workspace, workspace_bytes, stream);
}

int rb_st_search_shard(const float* query, int B, int D, const int64_t* probe_ids, int P,
                       const int64_t* cluster_offsets, const int64_t* cluster_sizes, int64_t n_lists, int64_t N,
                       int64_t pos_lo, int64_t pos_hi, const int8_t* item_codes, int k, int max_tensor_size_per_row,
                       int divisor_for_int8, const rb_st_filter* filter, uint64_t* out_pairs, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (out_pairs == nullptr) {
    set_last_error("st::search shard: out_pairs is required");
    return RB_ERR_INVALID_ARG;
  }
  return st_row_search(query, B, D, probe_ids, P, cluster_offsets, cluster_sizes, n_lists, N, pos_lo, pos_hi,
                       item_codes, nullptr, nullptr, k, max_tensor_size_per_row, divisor_for_int8, filter, nullptr,
                       nullptr, out_pairs, workspace, workspace_bytes, stream);
}

// Workspace of the grouped path: q codes [B, D] | q scales [B] | cnt, fill [L] int |
// cpo, ctask [L + 1] | pairs [B P] int32 | head, tail [B P] | row totals [B] |
// lists [B P, cap] | list counts [B P] | winner slots, raw [B, k_sel].
struct GroupWs {
  size_t codes, scales, cnt, fill, cpo, ctask, pairs, head, tail, total, lists, lcounts, slots, raw, bound, tc, err,
      bytes;
};

static GroupWs group_ws_layout(int B, int D, int P, int64_t n_lists, int k_sel) {
  GroupWs w;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += align_up(bytes, 256);
    return at;
  };
  const size_t pairs = static_cast<size_t>(B) * P;
  w.codes = take(static_cast<size_t>(B) * D);
  w.scales = take(static_cast<size_t>(B) * sizeof(float));
  w.cnt = take(static_cast<size_t>(n_lists) * sizeof(int));
  w.fill = take(static_cast<size_t>(n_lists) * sizeof(int));
  w.cpo = take(static_cast<size_t>(n_lists + 1) * sizeof(int64_t));
  w.ctask = take(static_cast<size_t>(n_lists + 1) * sizeof(int64_t));
  w.pairs = take(pairs * sizeof(int32_t));
  w.head = take(pairs * sizeof(int64_t));
  w.tail = take(pairs * sizeof(int64_t));
  w.total = take(static_cast<size_t>(B) * sizeof(int64_t));
  const int cap = std::max(group_cap(k_sel), ivf_tc_supported(D, k_sel, false) ? ivf_tc_cap(k_sel) : 0);
  w.lists = take(pairs * cap * sizeof(uint2));
  w.lcounts = take(pairs * sizeof(int));
  w.slots = take(static_cast<size_t>(B) * k_sel * sizeof(int64_t));
  w.raw = take(static_cast<size_t>(B) * k_sel * sizeof(float));
  w.bound = take(static_cast<size_t>(B) * sizeof(uint32_t));  // each row's bound on its k-th raw score
  // the tensor-core scan's gathered query blocks and task records, where it may run
  w.tc = take(ivf_tc_supported(D, k_sel, false) ? ivf_tc_ws_bytes(static_cast<int64_t>(B) * P, n_lists, D) : 0);
  w.err = take(256);  // the device error word of the tensor-core scan's bounded waits, last
  w.bytes = off;
  return w;
}

int rb_st_search_grouped_workspace_size(int B, int D, int P, int64_t n_lists, int k, int max_tensor_size_per_row,
                                        size_t* bytes) {
  if (bytes == nullptr || B < 0 || D <= 0 || P < 0 || n_lists < 0 || k < 1 || max_tensor_size_per_row < 0 ||
      max_tensor_size_per_row > INT32_MAX - 31) {
    set_last_error("st_search_grouped_workspace_size: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  const int width = st_width(max_tensor_size_per_row);
  *bytes = group_ws_layout(B, D, P, n_lists, std::max(std::min(k, width), 1)).bytes;  // as the search lays it out
  return RB_OK;
}

int rb_st_search_grouped(const float* query, int B, int D, const int64_t* probe_ids, int P,
                         const int64_t* cluster_offsets, const int64_t* cluster_sizes, int64_t n_lists,
                         const int8_t* item_codes, int64_t N, const int64_t* sort_perm, const float* global_scale,
                         int k, int max_tensor_size_per_row, int divisor_for_int8, const rb_st_filter* filter,
                         int64_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes,
                         void* stream) {
  int rc = st_check(B, D, P, n_lists, N, k, max_tensor_size_per_row, divisor_for_int8);
  if (rc != RB_OK) return rc;
  if (P > 1024 || static_cast<int64_t>(B) * P > INT32_MAX) {
    set_last_error("st::search (grouped): more than 1024 probes a row or 2^31 (row, probe) pairs");
    return RB_ERR_UNSUPPORTED;
  }
  FilterSet fs;
  rc = build_filters(filter, N, fs);
  if (rc != RB_OK) return rc;
  if (B == 0) return RB_OK;
  const int width = st_width(max_tensor_size_per_row);
  const int k_sel = std::min(k, width);
  const GroupWs lay = group_ws_layout(B, D, P, n_lists, std::max(k_sel, 1));
  if (workspace == nullptr || workspace_bytes < lay.bytes) {
    set_last_error("st::search: workspace too small");
    return RB_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int8_t* q_codes = reinterpret_cast<int8_t*>(ws + lay.codes);
  float* q_scales = reinterpret_cast<float*>(ws + lay.scales);
  rc = rb_quantize_int8(query, B, D, q_codes, q_scales, stream);
  if (rc != RB_OK) return rc;
  if (width == 0 || P == 0 || n_lists == 0) {
    fill_empty(out_ids, out_scores, static_cast<size_t>(B) * k, s);
    return launch_status();
  }
  int* cnt = reinterpret_cast<int*>(ws + lay.cnt);
  int* fill = reinterpret_cast<int*>(ws + lay.fill);
  int64_t* cpo = reinterpret_cast<int64_t*>(ws + lay.cpo);
  int64_t* ctask = reinterpret_cast<int64_t*>(ws + lay.ctask);
  int32_t* pairs = reinterpret_cast<int32_t*>(ws + lay.pairs);
  int64_t* head = reinterpret_cast<int64_t*>(ws + lay.head);
  int64_t* tail = reinterpret_cast<int64_t*>(ws + lay.tail);
  int64_t* total = reinterpret_cast<int64_t*>(ws + lay.total);
  uint2* lists = reinterpret_cast<uint2*>(ws + lay.lists);
  int* lcounts = reinterpret_cast<int*>(ws + lay.lcounts);
  int64_t* slots = reinterpret_cast<int64_t*>(ws + lay.slots);
  float* raw = reinterpret_cast<float*>(ws + lay.raw);
  const int64_t n_pairs = static_cast<int64_t>(B) * P;
  const bool bloom = fs.bloom.index != nullptr;
  const bool tc = ivf_tc_supported(D, k_sel, bloom);
  const int G = tc ? 128 : group_pairs_per_task(D);
  cudaMemsetAsync(cnt, 0, static_cast<size_t>(n_lists) * sizeof(int), s);
  cudaMemsetAsync(fill, 0, static_cast<size_t>(n_lists) * sizeof(int), s);
  cudaMemsetAsync(lcounts, 0, static_cast<size_t>(n_pairs) * sizeof(int), s);
  uint32_t* row_bound = reinterpret_cast<uint32_t*>(ws + lay.bound);
  cudaMemsetAsync(row_bound, 0, static_cast<size_t>(B) * sizeof(uint32_t), s);
  const int pgrid = static_cast<int>(std::min<int64_t>((n_pairs + 255) / 256, 4096));
  pair_count_kernel<<<pgrid, 256, 0, s>>>(probe_ids, n_pairs, n_lists, cnt);
  cluster_scan_kernel<<<1, kExpandThreads, 0, s>>>(cnt, n_lists, G, cpo, ctask);
  pair_scatter_kernel<<<pgrid, 256, 0, s>>>(probe_ids, n_pairs, n_lists, cpo, fill, pairs);
  slot_starts_kernel<<<(B + 127) / 128, 128, 0, s>>>(probe_ids, B, P, cluster_offsets, cluster_sizes, n_lists, N,
                                                      width, head, tail, total);
  rc = launch_status();
  if (rc != RB_OK) return rc;
  if (tc) {
    int* err = reinterpret_cast<int*>(ws + lay.err);
    cudaMemsetAsync(err, 0, sizeof(int), s);
    ProfileEvents& pe = profile_events();
    if (pe.start) record_profile_event(pe.start, s);
    rc = ivf_tc_scan(q_codes, B, D, P, item_codes, N, cluster_offsets, cluster_sizes, n_lists, pairs, cpo, ctask, head,
                     tail, width, k_sel, divisor_for_int8, fs, lists, lcounts, row_bound, err, ws + lay.tc, s);
    if (rc != RB_OK) return rc;
    if (pe.stop) record_profile_event(pe.stop, s);
  } else {
    rc = group_scan(item_codes, N, D, q_codes, probe_ids, P, cluster_offsets, cluster_sizes, n_lists, pairs, cpo,
                    ctask, head, tail, width, G, k_sel, divisor_for_int8, fs, lists, lcounts, row_bound, n_pairs, s);
    if (rc != RB_OK) return rc;
  }
  rc = merge_lists(lists, lcounts, B, P, tc ? ivf_tc_cap(k_sel) : group_cap(k_sel), k_sel, 0, slots, raw, nullptr, s);
  if (rc != RB_OK) return rc;
  const int64_t n = static_cast<int64_t>(B) * k;
  const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, 4096));
  st_group_epilogue_kernel<<<grid, 256, 0, s>>>(slots, raw, k_sel, probe_ids, P, cluster_offsets, cluster_sizes,
                                                n_lists, head, tail, total, width, sort_perm, N, q_scales,
                                                global_scale, divisor_for_int8, B, k, out_ids, out_scores);
  return launch_status();
}


static size_t finish_ws(int B, int D, int P, size_t* at) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t a = off;
    off += align_up(bytes, 256);
    return a;
  };
  at[0] = take(static_cast<size_t>(B) * D);                        // q codes
  at[1] = take(static_cast<size_t>(B) * sizeof(float));            // q scales
  at[2] = take(static_cast<size_t>(B) * P * sizeof(int64_t));      // head starts
  at[3] = take(static_cast<size_t>(B) * P * sizeof(int64_t));      // tail starts
  at[4] = take(static_cast<size_t>(B) * sizeof(int64_t));          // row totals
  return off;
}

int rb_st_search_finish_workspace_size(int B, int D, int P, size_t* bytes) {
  if (bytes == nullptr || B < 0 || D <= 0 || P < 0) {
    set_last_error("st_search_finish_workspace_size: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  size_t at[5];
  *bytes = finish_ws(B, D, P, at);
  return RB_OK;
}

int rb_st_search_finish(const float* query, int B, int D, const int64_t* probe_ids, int P,
                        const int64_t* cluster_offsets, const int64_t* cluster_sizes, int64_t n_lists, int64_t N,
                        const int64_t* sort_perm, const float* global_scale, int k, int max_tensor_size_per_row,
                        int divisor_for_int8, const int64_t* slots, const float* raw, int kin, int64_t* out_ids,
                        float* out_scores, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = st_check(B, D, P, n_lists, N, k, max_tensor_size_per_row, divisor_for_int8);
  if (rc != RB_OK) return rc;
  if (kin < 0 || kin > k) {
    set_last_error("st::search finish: the merged lists must hold at most k entries a row");
    return RB_ERR_INVALID_ARG;
  }
  if (B == 0) return RB_OK;
  size_t at[5];
  const size_t need = finish_ws(B, D, P, at);
  if (workspace == nullptr || workspace_bytes < need) {
    set_last_error("st::search finish: workspace too small");
    return RB_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* q_scales = reinterpret_cast<float*>(ws + at[1]);
  int64_t* head = reinterpret_cast<int64_t*>(ws + at[2]);
  int64_t* tail = reinterpret_cast<int64_t*>(ws + at[3]);
  int64_t* total = reinterpret_cast<int64_t*>(ws + at[4]);
  rc = rb_quantize_int8(query, B, D, reinterpret_cast<int8_t*>(ws + at[0]), q_scales, stream);
  if (rc != RB_OK) return rc;
  const int width = st_width(max_tensor_size_per_row);
  if (P > 0)
    slot_starts_kernel<<<(B + 127) / 128, 128, 0, s>>>(probe_ids, B, P, cluster_offsets, cluster_sizes, n_lists, N,
                                                        width, head, tail, total);
  const int64_t n = static_cast<int64_t>(B) * k;
  const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, 4096));
  st_group_epilogue_kernel<<<grid, 256, 0, s>>>(slots, raw, kin, probe_ids, P, cluster_offsets, cluster_sizes, n_lists,
                                                head, tail, total, width, sort_perm, N, q_scales, global_scale,
                                                divisor_for_int8, B, k, out_ids, out_scores);
  return launch_status();
}

int rb_st_fused_kmean_ann_workspace_size(int B, int P, int max_tensor_size_per_row, size_t* bytes) {
  if (bytes == nullptr || B < 0 || P < 0 || max_tensor_size_per_row < 0 || max_tensor_size_per_row > INT32_MAX - 31) {
    set_last_error("fused_kmean_ann_workspace_size: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  const int width = st_width(max_tensor_size_per_row);
  *bytes = align_up(static_cast<size_t>(B) * width * sizeof(int64_t), 256) +
           align_up(static_cast<size_t>(B) * sizeof(int64_t), 256);
  return RB_OK;
}

}  // extern "C"

// Block length of the float scorer's chains (simple_index_mm.cuh:237-300): the whole row when it
// fits 256 bytes, else 256 bytes' worth when that divides D, else 384 bytes' worth; 0 when
// neither divides D (the reference has no kernel for that D).
static int float_dot_unit(int D, int elem_bytes) {
  if (D % (16 / elem_bytes) != 0) return 0;
  if (D * elem_bytes <= 256) return D;
  if (D % (256 / elem_bytes) == 0) return 256 / elem_bytes;
  if (D % (384 / elem_bytes) == 0) return 384 / elem_bytes;
  return 0;
}

static int fused_kmean_ann_impl(const int64_t* cluster_offsets, int64_t n_lists, const int64_t* cluster_ids,
                                const int64_t* cluster_length, int P, const void* embeddings, int64_t N,
                                const void* queries, int dtype, int B, int D, int max_tensor_size_per_row,
                                const int64_t* filtering_bit_mask, int64_t mask_rows, int64_t mask_words,
                                const int64_t* filtering_bit_index, const PartialMask& pm,
                                const uint16_t* per_embedding_scale, int invalid_index_value, int divisor_for_int8,
                                void* out_raw, int32_t* out_idx, void* workspace, size_t workspace_bytes,
                                void* stream) {
  if (B < 0 || D <= 0 || P < 0 || n_lists < 0 || N < 0 || max_tensor_size_per_row < 0 ||
      max_tensor_size_per_row > INT32_MAX - 31 ||
      (filtering_bit_mask != nullptr && (mask_words < 0 || mask_rows < 0)) ||
      (filtering_bit_mask != nullptr && filtering_bit_index == nullptr && mask_rows < B) ||
      (divisor_for_int8 != -1 && divisor_for_int8 <= 0)) {
    set_last_error("fused_kmean_ann: bad sizes or divisor");
    return RB_ERR_INVALID_ARG;
  }
  if (P > kMaxProbes || B > 65535 || N > INT32_MAX || D > 16384) {
    set_last_error("fused_kmean_ann: more than 2048 probes, 65535 rows, 2^31 docs or D > 16384 is not supported");
    return RB_ERR_UNSUPPORTED;
  }
  if (dtype != RB_I8 && dtype != RB_F32 && dtype != RB_F16 && dtype != RB_BF16) {
    set_last_error("fused_kmean_ann: embeddings must be int8, fp32, fp16 or bf16");
    return RB_ERR_TYPE;
  }
  const int unit = dtype == RB_I8 ? D : float_dot_unit(D, dtype == RB_F32 ? 4 : 2);
  if (unit == 0) {
    set_last_error("fused_kmean_ann: D must be a multiple of 16 bytes, and past 256 bytes a multiple of 256 or "
                   "384 bytes, for float embeddings");
    return RB_ERR_UNSUPPORTED;
  }
  const int width = st_width(max_tensor_size_per_row);
  if (B == 0 || width == 0) return RB_OK;
  const size_t pos_bytes = align_up(static_cast<size_t>(B) * width * sizeof(int64_t), 256);
  if (workspace == nullptr || workspace_bytes < pos_bytes + align_up(static_cast<size_t>(B) * sizeof(int64_t), 256)) {
    set_last_error("fused_kmean_ann: workspace too small");
    return RB_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t* pos = static_cast<int64_t*>(workspace);
  int64_t* counts = reinterpret_cast<int64_t*>(static_cast<uint8_t*>(workspace) + pos_bytes);
  FilterSet fs{reinterpret_cast<const uint64_t*>(filtering_bit_mask), filtering_bit_mask ? mask_words : 0,
               ExactArgs{nullptr, 0, 0, nullptr, nullptr, nullptr, 0},
               BloomArgs{nullptr, 0, nullptr, 0, nullptr, 0, 0, nullptr, 0, 0},
               filtering_bit_mask ? filtering_bit_index : nullptr, mask_rows};
  const size_t smem = static_cast<size_t>(P) * (sizeof(int64_t) + 3 * sizeof(int));
  probe_expand_kernel<<<B, kExpandThreads, smem, s>>>(cluster_ids, P, cluster_offsets, nullptr, n_lists, N, fs, width,
                                                      0, N, pos, counts, cluster_length, pm);
  int rc = launch_status();
  if (rc != RB_OK) return rc;
  const dim3 grid(static_cast<unsigned>((width + 255) / 256), static_cast<unsigned>(B));
  if (dtype == RB_F32) {
    raw_scores_float_kernel<float><<<grid, 256, align_up(static_cast<size_t>(D) * 4, 16), s>>>(
        static_cast<const float*>(embeddings), N, D, unit, static_cast<const float*>(queries), pos, counts, width,
        invalid_index_value, -FLT_MAX, static_cast<float*>(out_raw), out_idx);
    return launch_status();
  }
  if (dtype == RB_F16) {
    raw_scores_float_kernel<__half><<<grid, 256, align_up(static_cast<size_t>(D) * 2, 16), s>>>(
        static_cast<const __half*>(embeddings), N, D, unit, static_cast<const __half*>(queries), pos, counts, width,
        invalid_index_value, __ushort_as_half(0xfbffu), static_cast<__half*>(out_raw), out_idx);
    return launch_status();
  }
  if (dtype == RB_BF16) {
    raw_scores_float_kernel<__nv_bfloat16><<<grid, 256, align_up(static_cast<size_t>(D) * 2, 16), s>>>(
        static_cast<const __nv_bfloat16*>(embeddings), N, D, unit, static_cast<const __nv_bfloat16*>(queries), pos,
        counts, width, invalid_index_value, __ushort_as_bfloat16(0xff7fu), static_cast<__nv_bfloat16*>(out_raw),
        out_idx);
    return launch_status();
  }
  const size_t qsm = align_up(static_cast<size_t>(D), 16);
  const int8_t* codes = static_cast<const int8_t*>(embeddings);
  const int8_t* qcodes = static_cast<const int8_t*>(queries);
  const __half* scale = reinterpret_cast<const __half*>(per_embedding_scale);
  if (divisor_for_int8 == -1 && scale == nullptr)
    raw_scores_kernel<false><<<grid, 256, qsm, s>>>(codes, N, D, qcodes, pos, counts, width, divisor_for_int8,
                                                    nullptr, invalid_index_value, out_raw, out_idx);
  else
    raw_scores_kernel<true><<<grid, 256, qsm, s>>>(codes, N, D, qcodes, pos, counts, width, divisor_for_int8,
                                                   scale, invalid_index_value, out_raw, out_idx);
  return launch_status();
}

extern "C" {

int rb_st_fused_kmean_ann(const int64_t* cluster_offsets, int64_t n_lists, const int64_t* cluster_ids,
                          const int64_t* cluster_length, int P, const void* embeddings, int64_t N,
                          const void* queries, int dtype, int B, int D, int max_tensor_size_per_row,
                          const int64_t* filtering_bit_mask, int64_t mask_rows, int64_t mask_words,
                          const int64_t* filtering_bit_index, const uint16_t* per_embedding_scale,
                          int invalid_index_value, int divisor_for_int8, void* out_raw, int32_t* out_idx,
                          void* workspace, size_t workspace_bytes, void* stream) {
  return fused_kmean_ann_impl(cluster_offsets, n_lists, cluster_ids, cluster_length, P, embeddings, N, queries, dtype,
                              B, D, max_tensor_size_per_row, filtering_bit_mask, mask_rows, mask_words,
                              filtering_bit_index,
                              PartialMask{nullptr, nullptr, nullptr, 0, 0}, per_embedding_scale, invalid_index_value,
                              divisor_for_int8, out_raw, out_idx, workspace, workspace_bytes, stream);
}

int rb_st_fused_kmean_ann_with_partial_masks(const int64_t* cluster_offsets, int64_t n_lists,
                                             const int64_t* cluster_ids, const int64_t* cluster_length, int P,
                                             const void* embeddings, int64_t N, const void* queries, int dtype,
                                             int B, int D,
                                             int max_tensor_size_per_row, const int32_t* column_counts_cumsum,
                                             const int8_t* first_item_offset_in_column,
                                             const int64_t* column_results, int64_t n_column_results,
                                             int64_t mask_rows, const int64_t* filtering_bit_index,
                                             const uint16_t* per_embedding_scale, int invalid_index_value,
                                             int divisor_for_int8, void* out_raw, int32_t* out_idx, void* workspace,
                                             size_t workspace_bytes, void* stream) {
  if (n_column_results < 0 || mask_rows < 0 ||
      (static_cast<int64_t>(B) * P > 0 &&
       (column_counts_cumsum == nullptr || first_item_offset_in_column == nullptr)) ||
      (n_column_results > 0 && column_results == nullptr) || (filtering_bit_index == nullptr && mask_rows < B)) {
    set_last_error("fused_kmean_ann_with_partial_masks: the partial mask needs its cumsum, offsets and words for "
                   "mask_rows x P ranges (mask_rows >= B without filtering_bit_index)");
    return RB_ERR_INVALID_ARG;
  }
  // an empty word array filters every doc out: partial_mask_pass never reads past n_words
  const PartialMask pm{column_counts_cumsum, first_item_offset_in_column,
                       reinterpret_cast<const uint64_t*>(column_results), n_column_results, P, filtering_bit_index,
                       mask_rows};
  return fused_kmean_ann_impl(cluster_offsets, n_lists, cluster_ids, cluster_length, P, embeddings, N, queries, dtype,
                              B, D, max_tensor_size_per_row, nullptr, 0, 0, nullptr, pm, per_embedding_scale,
                              invalid_index_value, divisor_for_int8, out_raw, out_idx, workspace, workspace_bytes,
                              stream);
}

int rb_st_probe_prep(const float* query, int B, int D, const int64_t* probe_ids, int P, const int64_t* cluster_offsets,
                     const int64_t* cluster_sizes, int64_t n_lists, int8_t* out_codes, float* out_scales,
                     int64_t* out_cluster_ids, int64_t* out_cluster_length, int64_t* out_cluster_offsets,
                     int32_t* out_warps, int32_t* out_rounded_cumsum, int32_t* out_remaining_cumsum,
                     int32_t* out_warp_cumsum, void* stream) {
  if (B < 0 || D <= 0 || P < 0 || n_lists < 0) {
    set_last_error("st::probe_prep: bad sizes");
    return RB_ERR_INVALID_ARG;
  }
  if (B == 0) return RB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = rb_quantize_int8(query, B, D, out_codes, out_scales, stream);
  if (rc != RB_OK || P == 0) return rc;
  const int64_t n = static_cast<int64_t>(B) * P;
  const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, 4096));
  probe_prep_gather_kernel<<<grid, 256, 0, s>>>(probe_ids, B, P, cluster_offsets, cluster_sizes, n_lists,
                                                out_cluster_ids, out_cluster_length, out_cluster_offsets, out_warps);
  probe_prep_row_cumsum_kernel<<<(B + 127) / 128, 128, 0, s>>>(out_cluster_length, B, P, out_rounded_cumsum);
  probe_prep_global_cumsum_kernel<<<1, kExpandThreads, 0, s>>>(out_cluster_length, n, out_remaining_cumsum,
                                                               out_warp_cumsum);
  return launch_status();
}

}  // extern "C"
