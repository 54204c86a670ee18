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
#include <algorithm>
#include <cstdint>

#include "rb_capi_internal.h"
#include "rb_common.cuh"

namespace rb {

constexpr int kExpandThreads = 256;
constexpr int kMaxProbes = 2048;  // per-probe table: 20 bytes a probe in shared memory
constexpr int kMaxSearchD = 1024;

__device__ __forceinline__ void probe_range(const int64_t* __restrict__ offsets, const int64_t* __restrict__ sizes,
                                            int64_t n_lists, int64_t N, int64_t c, int64_t& start, int64_t& len) {
  start = 0;
  len = 0;
  if (c < 0 || c >= n_lists) return;
  const int64_t s = offsets[c];
  const int64_t l = sizes[c];
  if (s < 0 || s >= N || l <= 0) return;
  start = s;
  len = l < N - s ? l : N - s;
}

// The exact clause filter (silvertorch/ops/csrc/fork_filters.cuh:15-41): attrs is the
// clause-major int32 [rows, docs] slot table, clause c in slots
// [clause_slots[c], clause_slots[c + 1]), each doc's values sorted descending with -1
// pads last; a clause with query value -1 passes, otherwise it matches when one of the
// doc's values equals the query's and passes when the match differs from reverse[c].
// Consecutive lanes test consecutive positions, so each slot row reads coalesced.
struct ExactArgs {
  const int32_t* attrs;  // null: no exact filter
  int64_t rows, docs;
  const int64_t* clause_slots;
  const uint8_t* reverse;
  const int32_t* query;  // [B, n_clauses]
  int n_clauses;
};

__device__ __forceinline__ bool exact_pass(const ExactArgs& ex, const int32_t* __restrict__ q, int64_t doc) {
  for (int c = 0; c < ex.n_clauses; ++c) {
    const int32_t qv = q[c];
    if (qv == -1) continue;
    bool match = false;
    const int64_t s1 = min(ex.clause_slots[c + 1], ex.rows);
    for (int64_t s = max(ex.clause_slots[c], int64_t{0}); s < s1; ++s) {
      const int32_t v = ex.attrs[s * ex.docs + doc];
      if (v == qv || v == -1) {
        match = v == qv;
        break;
      }
    }
    if (match == (ex.reverse[c] != 0)) return false;
  }
  return true;
}

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
    const int64_t* __restrict__ sizes, int64_t n_lists, int64_t N, const uint64_t* __restrict__ mask,
    int64_t mask_words, ExactArgs ex, int width, int64_t* __restrict__ pos, int64_t* __restrict__ counts) {
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
  const uint64_t* mrow = mask ? mask + static_cast<int64_t>(b) * mask_words : nullptr;
  const int32_t* qattrs = ex.attrs ? ex.query + static_cast<int64_t>(b) * ex.n_clauses : nullptr;
  auto emit = [&](int64_t slot, int64_t position) {
    if (slot >= width) return;
    int64_t v = position;
    if (mrow != nullptr) {
      const int64_t w = position >> 6;
      if (w < mask_words && ((mrow[w] >> (63 - (position & 63))) & 1ull) == 0) v = -1;
    }
    if (qattrs != nullptr && v >= 0 && !exact_pass(ex, qattrs, position)) v = -1;
    out[slot] = v;
  };
  for (int j = warp; j < P; j += kExpandThreads / 32) {
    const int64_t start = p_start[j];
    const int len = p_len[j];
    const int full = len / 32 * 32;
    const int64_t hs = p_head[j], ts = p_tail[j];
    for (int i = lane; i < full; i += 32) emit(hs + i, start + i);
    for (int i = lane; i < len - full; i += 32) emit(ts + i, start + full + i);
  }
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
  w.cand = take(cand_i8_ws_bytes(B, width));
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
    set_last_error("st::search: min(k, padded width) > 224 is not supported");
    return RB_ERR_UNSUPPORTED;
  }
  return RB_OK;
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

int rb_st_search(const float* query, int B, int D, const int64_t* probe_ids, int P, const int64_t* cluster_offsets,
                 const int64_t* cluster_sizes, int64_t n_lists, const int8_t* item_codes, int64_t N,
                 const int64_t* sort_perm, const float* global_scale, int k, int max_tensor_size_per_row,
                 int divisor_for_int8, const int64_t* filtering_bit_mask, int64_t mask_words,
                 const int32_t* item_clause_attrs, int64_t attr_rows, int64_t attr_docs, const int64_t* clause_slots,
                 const uint8_t* clause_is_reverse, const int32_t* query_clause_attrs, int n_clauses,
                 int64_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = st_check(B, D, P, n_lists, N, k, max_tensor_size_per_row, divisor_for_int8);
  if (rc != RB_OK) return rc;
  if (filtering_bit_mask != nullptr && mask_words < 0) {
    set_last_error("st::search: bad filtering_bit_mask width");
    return RB_ERR_INVALID_ARG;
  }
  ExactArgs ex{nullptr, 0, 0, nullptr, nullptr, nullptr, 0};
  if (query_clause_attrs != nullptr) {
    if (filtering_bit_mask != nullptr) {
      set_last_error("st::search takes one filter: the exact clauses or filtering_bit_mask");
      return RB_ERR_INVALID_ARG;
    }
    if (item_clause_attrs == nullptr || clause_slots == nullptr || clause_is_reverse == nullptr || n_clauses < 0 ||
        attr_rows < 0 || attr_docs < N) {
      set_last_error("st::search: the exact filter needs item_clause_attrs [R, >= N], clause_slots and "
                     "clause_is_reverse");
      return RB_ERR_INVALID_ARG;
    }
    ex = ExactArgs{item_clause_attrs, attr_rows, attr_docs, clause_slots, clause_is_reverse, query_clause_attrs,
                   n_clauses};
  }
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
    fill_empty(out_ids, out_scores, static_cast<size_t>(B) * k, s);
    return launch_status();
  }
  const size_t smem = static_cast<size_t>(P) * (sizeof(int64_t) + 3 * sizeof(int));
  probe_expand_kernel<<<B, kExpandThreads, smem, s>>>(
      probe_ids, P, cluster_offsets, cluster_sizes, n_lists, N, reinterpret_cast<const uint64_t*>(filtering_bit_mask),
      mask_words, ex, width, pos, counts);
  rc = launch_status();
  if (rc != RB_OK) return rc;
  rc = cand_i8_topk(q_codes, item_codes, static_cast<int>(N), D, pos, width, counts, B, k_sel, divisor_for_int8,
                    slots, raw, ws + lay.cand, s);
  if (rc != RB_OK) return rc;
  const int64_t n = static_cast<int64_t>(B) * k;
  const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, 4096));
  st_epilogue_kernel<<<grid, 256, 0, s>>>(slots, raw, k_sel, pos, counts, width, sort_perm, N, q_scales, global_scale,
                                          divisor_for_int8, B, k, out_ids, out_scores);
  return launch_status();
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
