// extern "C" entry points of libretrieve_b200: argument checks, workspace
// carving and the sequence of kernel launches for each op.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <string>

#include "rb_capi_internal.h"

namespace rb {

static thread_local std::string g_last_error;

void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }

ProfileEvents& profile_events() {
  static thread_local ProfileEvents ev;
  return ev;
}

static int fail(int code, const char* msg) {
  set_last_error(msg);
  return code;
}
static int fail(int code, const std::string& msg) { return fail(code, msg.c_str()); }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Records a profiling event; inside a CUDA graph capture as an event record
// node, so that every replay of the graph records it.
void record_profile_event(cudaEvent_t ev, cudaStream_t stream) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &st) == cudaSuccess && st == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(ev, stream, cudaEventRecordExternal);
  else
    cudaEventRecord(ev, stream);
}

// Workspace tail: one device error word, 256-byte aligned at the end.
static int* ws_err_word(void* ws, size_t ws_bytes) {
  return reinterpret_cast<int*>(static_cast<uint8_t*>(ws) + ws_bytes - 256);
}

}  // namespace rb

using namespace rb;

extern "C" {

const char* rb_last_error(void) { return g_last_error.c_str(); }

int rb_abi_version(void) { return 2; }

int rb_dense_topk_workspace_size(int B, int N, int D, int dtype, int k, size_t* bytes) {
  if (bytes == nullptr) return fail(RB_ERR_INVALID_ARG, "bytes is null");
  if (B < 0 || N < 0 || D <= 0 || k < 1) return fail(RB_ERR_INVALID_ARG, "dense_topk: bad shape or k");
  *bytes = dense_workspace_bytes(B, N, k, dense_row_bytes(D, dtype), dense_scaled(dtype));
  return RB_OK;
}

// Shared body of the dense entry points (elem 0 f16, 1 bf16, 2 int8).
// Threshold shared by the shards of a row-sharded search: seed_vals is the
// [W, B, k] stack of every shard's rb_dense_seed_sample output and n_total the
// corpus size over all shards.
struct SharedSeed {
  const float* vals;  // [W, B, m]
  int W, m;
  int64_t n_total;
};

static int dense_check(int elem, const void* queries, const float* q_scale, const void* items, const float* x_scale,
                       int B, int N, int D, int k, const char* what) {
  if (B < 0 || N < 0 || k < 1) return fail(RB_ERR_INVALID_ARG, std::string(what) + ": bad B, N or k");
  if (k > 1024) return fail(RB_ERR_UNSUPPORTED, std::string(what) + ": k > 1024 is not supported");
  const int row_bytes = (elem == 2 || elem == 4) ? D : 2 * D;
  if (row_bytes != 128 && row_bytes != 256 && row_bytes != 512)
    return fail(RB_ERR_UNSUPPORTED, std::string(what) +
                                        ": rows must be 128, 256 or 512 bytes (D = 64/128/256 fp16/bf16, "
                                        "128/256/512 int8)");
  if (B > 0 && N > 0) {
    if (!aligned16(queries) || !aligned16(items)) return fail(RB_ERR_INVALID_ARG, std::string(what) + ": 16-byte alignment");
    if (elem >= 2 && x_scale != nullptr && !aligned16(x_scale))
      return fail(RB_ERR_INVALID_ARG, std::string(what) + ": item scales must be 16-byte aligned");
  }
  return RB_OK;
}

// After a pass from the speculative seed: a row whose k-th output is padding found fewer
// than k candidates at or above that seed, and is scanned again from the safe seed (the
// k-th sampled tile max); every other row keeps its output (seed NaN: nothing passes).
__global__ void spec_check_kernel(const int64_t* __restrict__ out_ids, int B, int k, const float* __restrict__ safe,
                                  float* __restrict__ seed, int* __restrict__ row_live, int* __restrict__ qsg_live,
                                  int queries_per_group) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= B) return;
  // (a row whose safe seed is no lower, e.g. both -inf, already ran from the safe seed)
  const bool again = out_ids[static_cast<int64_t>(q) * k + (k - 1)] < 0 && safe[q] < seed[q];
  row_live[q] = again ? 1 : 0;
  seed[q] = again ? safe[q] : __int_as_float(0x7fc00000);
  if (again) atomicOr(&qsg_live[q / queries_per_group], 1);
}

// The same for batches of more than kSpecRows rows, one block: the first kSpecRows short rows
// (in row order) go to fail_rows for the compact second pass; any further ones are marked for
// the pass over their query groups (row_live, seed, qsg_live) as spec_check_kernel does.
// fail_rows is padded with -1; *c_live says whether the compact pass has a row.
__global__ void __launch_bounds__(1024) spec_select_kernel(const int64_t* __restrict__ out_ids, int B, int k,
                                                           const float* __restrict__ safe, float* __restrict__ seed,
                                                           int* __restrict__ row_live, int* __restrict__ qsg_live,
                                                           int queries_per_group, int* __restrict__ fail_rows,
                                                           int* __restrict__ c_live) {
  __shared__ int warp_count[32];
  __shared__ int found;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (threadIdx.x == 0) found = 0;
  __syncthreads();
  for (int q0 = 0; q0 < B; q0 += blockDim.x) {
    const int q = q0 + static_cast<int>(threadIdx.x);
    const bool again = q < B && out_ids[static_cast<int64_t>(q) * k + (k - 1)] < 0 && safe[q] < seed[q];
    const uint32_t bal = __ballot_sync(RB_FULL_MASK, again);
    if (lane == 0) warp_count[w] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) {
      before += i < w ? warp_count[i] : 0;
      total += warp_count[i];
    }
    const int pos = found + before + __popc(bal & lanemask_lt());
    if (q < B) {
      if (again && pos < kSpecRows) {
        fail_rows[pos] = q;  // the compact pass takes it
        row_live[q] = 0;
        seed[q] = __int_as_float(0x7fc00000);
      } else if (again) {
        row_live[q] = 1;
        seed[q] = safe[q];
        atomicOr(&qsg_live[q / queries_per_group], 1);
      } else {
        row_live[q] = 0;
        seed[q] = __int_as_float(0x7fc00000);
      }
    }
    __syncthreads();  // every thread has read `found` and warp_count
    if (threadIdx.x == 0) found += total;
    __syncthreads();
  }
  for (int c = found + static_cast<int>(threadIdx.x); c < kSpecRows; c += blockDim.x) fail_rows[c] = -1;
  if (threadIdx.x == 0) *c_live = found > 0 ? 1 : 0;
}

// Row c of the compact batch: short row fail_rows[c]'s query, query scale, safe seed and
// predicate terms (zero query, NaN seed and no terms for a padding row).
__global__ void spec_gather_kernel(const int* __restrict__ fail_rows, const uint8_t* __restrict__ queries,
                                   int row_bytes, const float* __restrict__ q_scale, const float* __restrict__ safe,
                                   const PredTerm* __restrict__ terms, const int* __restrict__ n_terms,
                                   uint8_t* __restrict__ qc, float* __restrict__ qsc, float* __restrict__ seedc,
                                   PredTerm* __restrict__ termsc, int* __restrict__ ntc, int* __restrict__ row_live_c) {
  const int c = blockIdx.x;
  const int src = fail_rows[c];
  const int n16 = row_bytes / 16;
  int4* dst = reinterpret_cast<int4*>(qc + static_cast<size_t>(c) * row_bytes);
  const int4* from = reinterpret_cast<const int4*>(queries + static_cast<size_t>(src < 0 ? 0 : src) * row_bytes);
  for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src >= 0 ? from[i] : make_int4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    qsc[c] = (src >= 0 && q_scale != nullptr) ? q_scale[src] : 1.f;
    seedc[c] = src >= 0 ? safe[src] : __int_as_float(0x7fc00000);
    row_live_c[c] = src >= 0 ? 1 : 0;
    if (terms != nullptr) ntc[c] = src >= 0 ? n_terms[src] : 0;
  }
  if (terms != nullptr && static_cast<int>(threadIdx.x) < kMaxTerms)
    termsc[c * kMaxTerms + threadIdx.x] =
        src >= 0 ? terms[static_cast<size_t>(src) * kMaxTerms + threadIdx.x] : PredTerm{0, 0, 0, 0};
}

// The compact pass's results back to their rows.
__global__ void spec_scatter_kernel(const int* __restrict__ fail_rows, int k, const int64_t* __restrict__ idsc,
                                    const float* __restrict__ scoresc, int64_t* __restrict__ out_ids,
                                    float* __restrict__ out_scores) {
  const int c = blockIdx.x;
  const int src = fail_rows[c];
  if (src < 0) return;
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    out_ids[static_cast<int64_t>(src) * k + j] = idsc[static_cast<int64_t>(c) * k + j];
    out_scores[static_cast<int64_t>(src) * k + j] = scoresc[static_cast<int64_t>(c) * k + j];
  }
}

// The rank F k / s of the speculative seed among the sampled tile maxima (dense_topk_impl).
// Every epilogue costs in proportion to the chunks that reach the threshold: from the safe
// seed (rank about k s) the plain fp16 / bf16 pass appends in about half of its 32 x 128
// warp-tiles, and those appends, not the MMA, set its pace. F = 3 for every scan (measured
// at 10M items: bf16 2.02 ms a search against 2.39 from the safe seed and 2.07 at F = 4; the
// filtered pass at 10 % selectivity 4.8 ms at F = 3 against 5.4 at F = 2, where the compact
// second pass ran in every batch, and at F = 4; int8 38.2 ms at F = 3 against 40.5 at F = 2).
static bool dense_spec_applies(int elem, const FilterArgs* filter) {
  (void)elem;
  (void)filter;
  return true;
}
static int dense_spec_factor(const FilterArgs* filter) {
  (void)filter;
  return 3;
}
static int dense_spec_rank(int k, const DensePlan& pl, int factor) {
  return static_cast<int>((static_cast<int64_t>(factor) * k + pl.sample_stride - 1) / pl.sample_stride);
}

struct DenseWs {
  uint2* lists;
  int* counts;
  float* thresh;
  int* err;
};

// The layout of dense_workspace_bytes: the candidate lists share their region with the
// sampling pass's tile maxima, so the counts and seeds start past the larger of the two
// (the seeds are written while the tile maxima are still being read).
static DenseWs dense_ws(void* workspace, size_t workspace_bytes, int B, const DensePlan& pl) {
  DenseWs d;
  uint8_t* w = static_cast<uint8_t*>(workspace);
  d.lists = reinterpret_cast<uint2*>(w);
  const size_t lists = static_cast<size_t>(B) * pl.n_lists * pl.cap * sizeof(uint2);
  const size_t cm = static_cast<size_t>(B) * dense_chunk_stride(pl) * sizeof(float);
  w += align_up(std::max(lists, cm), 256);
  d.counts = reinterpret_cast<int*>(w);
  w += align_up(static_cast<size_t>(B) * pl.n_lists * sizeof(int), 256);
  d.thresh = reinterpret_cast<float*>(w);
  d.err = ws_err_word(workspace, workspace_bytes);
  return d;
}

// The compact second pass's buffers, after the seeds: kSpecRows query rows (up to 512 bytes)
// | their terms | ids | scores [kSpecRows, k] | row indices, query scales, seeds, term counts,
// row flags (kSpecRows each) | the pass's live flag (dense_workspace_bytes reserves them).
struct SpecWs {
  uint8_t* queries;
  PredTerm* terms;
  int64_t* ids;
  float* scores;
  int* fail_rows;
  float* q_scale;
  float* seed;
  int* n_terms;
  int* row_live;
  int* live;
};

static SpecWs spec_ws(const DenseWs& d, int B, const DensePlan& pl, int k) {
  (void)pl;
  uint8_t* w = reinterpret_cast<uint8_t*>(d.thresh) + align_up((4 * static_cast<size_t>(B) + 64) * sizeof(float), 256);
  SpecWs c;
  auto take = [&](size_t bytes) {
    uint8_t* at = w;
    w += align_up(bytes, 256);
    return at;
  };
  c.queries = take(static_cast<size_t>(kSpecRows) * 512);
  c.terms = reinterpret_cast<PredTerm*>(take(static_cast<size_t>(kSpecRows) * kMaxTerms * sizeof(PredTerm)));
  c.ids = reinterpret_cast<int64_t*>(take(static_cast<size_t>(kSpecRows) * k * sizeof(int64_t)));
  c.scores = reinterpret_cast<float*>(take(static_cast<size_t>(kSpecRows) * k * sizeof(float)));
  c.fail_rows = reinterpret_cast<int*>(take(kSpecRows * sizeof(int)));
  c.q_scale = reinterpret_cast<float*>(take(kSpecRows * sizeof(float)));
  c.seed = reinterpret_cast<float*>(take(kSpecRows * sizeof(float)));
  c.n_terms = reinterpret_cast<int*>(take(kSpecRows * sizeof(int)));
  c.row_live = reinterpret_cast<int*>(take(kSpecRows * sizeof(int)));
  c.live = reinterpret_cast<int*>(take(sizeof(int)));
  return c;
}

static int dense_topk_impl(int elem, const void* queries, const float* q_scale, const void* items,
                           const float* x_scale, int B, int N, int D, int k, int64_t id_offset, int64_t* out_ids,
                           float* out_scores, void* workspace, size_t workspace_bytes, cudaStream_t stream,
                           const FilterArgs* filter = nullptr, const SharedSeed* shared = nullptr,
                           uint2* out_pairs = nullptr) {
  int rc = dense_check(elem, queries, q_scale, items, x_scale, B, N, D, k, "dense_topk");
  if (rc != RB_OK) return rc;
  if (B == 0) return RB_OK;
  if (out_pairs == nullptr && (out_ids == nullptr || out_scores == nullptr))
    return fail(RB_ERR_INVALID_ARG, "dense_topk: null output");
  if (N == 0) {
    if (out_pairs != nullptr) fill_empty_pairs(out_pairs, static_cast<size_t>(B) * k, stream);
    else fill_empty(out_ids, out_scores, static_cast<size_t>(B) * k, stream);
    return cudaGetLastError() == cudaSuccess ? RB_OK : fail(RB_ERR_CUDA, "fill_empty launch failed");
  }
  const int row_bytes = (elem == 2 || elem == 4) ? D : 2 * D;
  if (filter != nullptr && (k > 384 || row_bytes > 256))
    return fail(RB_ERR_UNSUPPORTED, "dense_topk_filtered: k <= 384 and rows of up to 256 bytes");
  const size_t need = dense_workspace_bytes(B, N, k, row_bytes, elem >= 2);
  if (workspace == nullptr || workspace_bytes < need) return fail(RB_ERR_WORKSPACE, "dense_topk: workspace too small");
  // A Bloom filter with room for its bit-sliced words (rb_dense_topk_filtered_workspace_size):
  // they go where a workspace of exactly `need` bytes keeps its error word, and the scans
  // test 32 items per term and AND. A smaller workspace keeps the per-item test.
  FilterArgs sliced_filter;
  if (filter != nullptr && (filter->mode == kFilterBloom || filter->mode == kFilterBloomRecheck) &&
      filter->slices == nullptr && workspace_bytes >= need + bloom_slices_bytes(N)) {
    sliced_filter = *filter;
    uint32_t* slices = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + need - 256);
    if (bloom_slices(filter->bloom, N, slices, stream) != RB_OK) return fail(RB_ERR_CUDA, "bloom slices launch failed");
    sliced_filter.slices = slices;
    filter = &sliced_filter;
  }

  DensePlan pl;
  dense_plan(B, N, k, row_bytes, pl, shared ? shared->n_total : N, elem >= 2);
  const DenseWs d = dense_ws(workspace, workspace_bytes, B, pl);
  if (cudaMemsetAsync(d.err, 0, sizeof(int), stream) != cudaSuccess) return fail(RB_ERR_CUDA, "memset failed");

  ProfileEvents& pe = profile_events();
  const float* seed = nullptr;
  // Filtered and int8 searches start the full pass from a speculative seed: the
  // ceil(F k / s)-th largest sampled tile max instead of the k-th (s = the sample's tile
  // stride). About F k items of the corpus reach it (a count whose spread is about
  // 1 / sqrt(F k / s)), so the rows test about s / F times fewer candidates; a row that still
  // finds fewer than k runs again from the safe seed, in the compact batch of up to 128 such
  // rows or, past those, with its query group.
  bool spec = false;
  if (shared != nullptr) {
    // k-th largest of the union of the shards' samples (a [W, B, k] stack)
    rc = row_kth_lower_bound(shared->vals, B, shared->m, shared->m, shared->W, static_cast<int64_t>(B) * shared->m,
                             k, d.thresh, nullptr, stream);
    if (rc != RB_OK) return rc;
    seed = d.thresh;
  } else if (pl.sample_stride > 0) {
    float* chunk_max = reinterpret_cast<float*>(d.lists);  // dead before the full pass writes lists
    rc = dense_scan_pass(1, elem, queries, items, B, N, D, pl, k, nullptr, d.lists, d.counts, chunk_max, d.err,
                         stream, q_scale, x_scale, filter);
    if (rc != RB_OK) return rc;
    const int n_chunks = static_cast<int>(dense_chunk_stride(pl));
    const int k_spec = dense_spec_rank(k, pl, dense_spec_factor(filter));
    spec = dense_spec_applies(elem, filter) && out_pairs == nullptr && k_spec < k;
    if (spec)  // the speculative seed, and the safe one kept for the rows that need a second pass
      rc = row_kth2_lower_bounds(chunk_max, B, n_chunks, n_chunks, k_spec, k, d.thresh, d.thresh + B, stream);
    else
      rc = row_kth_lower_bound(chunk_max, B, n_chunks, n_chunks, 1, 0, k, d.thresh, nullptr, stream);
    if (rc != RB_OK) return rc;
    seed = d.thresh;
  }
  if (pe.start) record_profile_event(pe.start, stream);
  rc = dense_scan_pass(0, elem, queries, items, B, N, D, pl, k, seed, d.lists, d.counts, nullptr, d.err, stream,
                       q_scale, x_scale, filter);
  if (rc != RB_OK) return rc;
  if (pe.stop) record_profile_event(pe.stop, stream);  // the profiled span: the full pass alone
  if (!spec) {
    return merge_lists(d.lists, d.counts, B, pl.n_lists, pl.cap, k, id_offset, out_ids, out_scores, out_pairs,
                       stream);
  }
  rc = merge_lists(d.lists, d.counts, B, pl.n_lists, pl.cap, k, id_offset, out_ids, out_scores, nullptr, stream);
  if (rc != RB_OK) return rc;
  int* row_live = reinterpret_cast<int*>(d.thresh + 2 * static_cast<size_t>(B));
  int* qsg_live = reinterpret_cast<int*>(d.thresh + 3 * static_cast<size_t>(B));
  if (cudaMemsetAsync(qsg_live, 0, static_cast<size_t>(pl.n_qsg) * sizeof(int), stream) != cudaSuccess)
    return fail(RB_ERR_CUDA, "memset failed");
  // queries of one query group: ng MMA tiles of 128 rows, doubled across a CTA pair
  const int per_group = pl.ng * (pl.two_sm ? 256 : 128);
  if (B <= kSpecRows) {
    spec_check_kernel<<<(B + 255) / 256, 256, 0, stream>>>(out_ids, B, k, d.thresh + B, d.thresh, row_live,
                                                           qsg_live, per_group);
    if (cudaGetLastError() != cudaSuccess) return fail(RB_ERR_CUDA, "spec_check launch failed");
  } else {
    // Up to kSpecRows short rows run again as one compact 128-row batch on the 1-SM kernel
    // (their queries, scales, seeds and terms gathered), its lists in the main lists region.
    const SpecWs c = spec_ws(d, B, pl, k);
    spec_select_kernel<<<1, 1024, 0, stream>>>(out_ids, B, k, d.thresh + B, d.thresh, row_live, qsg_live,
                                               per_group, c.fail_rows, c.live);
    const int row_bytes_q = (elem == 2 || elem == 4) ? D : 2 * D;
    FilterArgs fc{};
    if (filter != nullptr) fc = *filter;
    spec_gather_kernel<<<kSpecRows, 128, 0, stream>>>(
        c.fail_rows, static_cast<const uint8_t*>(queries), row_bytes_q, q_scale, d.thresh + B,
        filter != nullptr ? filter->terms : nullptr, filter != nullptr ? filter->n_terms : nullptr, c.queries,
        c.q_scale, c.seed, c.terms, c.n_terms, c.row_live);
    if (cudaGetLastError() != cudaSuccess) return fail(RB_ERR_CUDA, "spec gather launch failed");
    fc.terms = c.terms;
    fc.n_terms = c.n_terms;
    DensePlan pc;
    dense_plan(kSpecRows, N, k, row_bytes_q, pc, N, elem >= 2);
    // as many splits as the main lists region (and counts region) holds
    const size_t region = align_up(std::max(static_cast<size_t>(B) * pl.n_lists * pl.cap * sizeof(uint2),
                                            static_cast<size_t>(B) * dense_chunk_stride(pl) * sizeof(float)),
                                   256);
    const int64_t fit_lists = static_cast<int64_t>(region / (static_cast<size_t>(kSpecRows) * pc.cap * sizeof(uint2)));
    const int64_t fit_counts = static_cast<int64_t>(B) * pl.n_lists / kSpecRows;
    pc.n_splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({fit_lists, fit_counts, pc.n_splits})));
    pc.n_lists = pc.n_splits;
    rc = dense_scan_pass(0, elem, c.queries, items, kSpecRows, N, D, pc, k, c.seed, d.lists, d.counts, nullptr, d.err,
                         stream, q_scale != nullptr ? c.q_scale : nullptr, x_scale, filter != nullptr ? &fc : nullptr,
                         c.live);
    if (rc != RB_OK) return rc;
    rc = merge_lists(d.lists, d.counts, kSpecRows, pc.n_lists, pc.cap, k, id_offset, c.ids, c.scores, nullptr, stream,
                     c.row_live);
    if (rc != RB_OK) return rc;
    spec_scatter_kernel<<<kSpecRows, 128, 0, stream>>>(c.fail_rows, k, c.ids, c.scores, out_ids, out_scores);
    if (cudaGetLastError() != cudaSuccess) return fail(RB_ERR_CUDA, "spec scatter launch failed");
  }
  // the rows left scan again with their query groups (no group: every task skipped)
  rc = dense_scan_pass(0, elem, queries, items, B, N, D, pl, k, d.thresh, d.lists, d.counts, nullptr, d.err, stream,
                       q_scale, x_scale, filter, qsg_live);
  if (rc != RB_OK) return rc;
  return merge_lists(d.lists, d.counts, B, pl.n_lists, pl.cap, k, id_offset, out_ids, out_scores, nullptr, stream,
                     row_live);
}

int rb_dense_seed_sample(const void* queries, const void* items, int B, int N, int D, int dtype, int k, int m,
                         int64_t n_total, float* out_vals, void* workspace, size_t workspace_bytes, void* stream_) {
  if (dtype != RB_F16 && dtype != RB_BF16) return fail(RB_ERR_TYPE, "dense_seed_sample: dtype must be f16 or bf16");
  const int elem = dtype == RB_BF16 ? 1 : 0;
  int rc = dense_check(elem, queries, nullptr, items, nullptr, B, N, D, k, "dense_seed_sample");
  if (rc != RB_OK) return rc;
  if (B == 0) return RB_OK;
  if (out_vals == nullptr) return fail(RB_ERR_INVALID_ARG, "dense_seed_sample: null output");
  if (m < 1 || m > k) return fail(RB_ERR_INVALID_ARG, "dense_seed_sample: need 1 <= m <= k");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const size_t need = dense_workspace_bytes(B, N, k, 2 * D);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(RB_ERR_WORKSPACE, "dense_seed_sample: workspace too small");
  DensePlan pl;
  dense_plan(B, N, k, 2 * D, pl, std::max<int64_t>(n_total, N));
  const DenseWs d = dense_ws(workspace, workspace_bytes, B, pl);
  if (N == 0 || pl.sample_stride == 0) {
    // nothing sampled on this shard: m times -inf per query
    return row_kth_lower_bound(nullptr, B, 0, 0, 1, 0, m, d.thresh, out_vals, stream);
  }
  if (cudaMemsetAsync(d.err, 0, sizeof(int), stream) != cudaSuccess) return fail(RB_ERR_CUDA, "memset failed");
  float* chunk_max = reinterpret_cast<float*>(d.lists);
  rc = dense_scan_pass(1, elem, queries, items, B, N, D, pl, k, nullptr, d.lists, d.counts, chunk_max, d.err, stream,
                       nullptr, nullptr, nullptr);
  if (rc != RB_OK) return rc;
  const int n_chunks = static_cast<int>(dense_chunk_stride(pl));
  // m values at or above the shard's m-th largest tile max: its top m, up to
  // the 22-bit rounding of the bound
  return row_kth_lower_bound(chunk_max, B, n_chunks, n_chunks, 1, 0, m, d.thresh, out_vals, stream);
}

int rb_dense_topk_seeded(const void* queries, const void* items, int B, int N, int D, int dtype, int k,
                         int64_t id_offset, int64_t n_total, const float* seed_vals, int W, int m, int64_t* out_ids,
                         float* out_scores, uint64_t* out_pairs, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (dtype != RB_F16 && dtype != RB_BF16) return fail(RB_ERR_TYPE, "dense_topk_seeded: dtype must be f16 or bf16");
  if (seed_vals == nullptr || W < 1 || m < 1 || m > k)
    return fail(RB_ERR_INVALID_ARG, "dense_topk_seeded: seed values missing or 1 <= m <= k violated");
  if (out_pairs != nullptr && (id_offset < 0 || id_offset + static_cast<int64_t>(N) > 0xffffffffll))
    return fail(RB_ERR_UNSUPPORTED, "dense_topk_seeded: pair output needs global ids below 2^32 - 1");
  const SharedSeed shared{seed_vals, W, m, std::max<int64_t>(n_total, N)};
  return dense_topk_impl(dtype == RB_BF16 ? 1 : 0, queries, nullptr, items, nullptr, B, N, D, k, id_offset, out_ids,
                         out_scores, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), nullptr, &shared,
                         reinterpret_cast<uint2*>(out_pairs));
}

int rb_merge_pairs(const uint64_t* pairs, int W, int B, int kin, int k, int64_t* out_ids, float* out_scores,
                   void* stream) {
  if (W < 1 || B < 0 || kin < 1 || k < 1) return fail(RB_ERR_INVALID_ARG, "merge_pairs: bad arguments");
  if (k > 1024) return fail(RB_ERR_UNSUPPORTED, "merge_pairs: k > 1024");
  if (W > 1024) return fail(RB_ERR_UNSUPPORTED, "merge_pairs: more than 1024 shards");
  if (B == 0) return RB_OK;
  if (pairs == nullptr || out_ids == nullptr || out_scores == nullptr)
    return fail(RB_ERR_INVALID_ARG, "merge_pairs: null pointer");
  return merge_pair_stack(reinterpret_cast<const uint2*>(pairs), W, B, kin, k, out_ids, out_scores,
                          static_cast<cudaStream_t>(stream));
}

int rb_dense_topk(const void* queries, const void* items, int B, int N, int D, int dtype, int k, int64_t id_offset,
                  int64_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != RB_F16 && dtype != RB_BF16) return fail(RB_ERR_TYPE, "dense_topk: dtype must be f16 or bf16");
  return dense_topk_impl(dtype == RB_BF16 ? 1 : 0, queries, nullptr, items, nullptr, B, N, D, k, id_offset, out_ids,
                         out_scores, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int rb_dense_topk_filtered_workspace_size(int B, int N, int D, int dtype, int k, int mode, size_t* bytes) {
  const int rc = rb_dense_topk_workspace_size(B, N, D, dtype, k, bytes);
  if (rc != RB_OK) return rc;
  if (mode < RB_FILTER_NONE || mode > RB_FILTER_BLOOM_RECHECK)
    return fail(RB_ERR_INVALID_ARG, "dense_topk_filtered_workspace_size: unknown filter mode");
  if (mode == RB_FILTER_BLOOM || mode == RB_FILTER_BLOOM_RECHECK) *bytes += bloom_slices_bytes(N);
  return RB_OK;
}

int rb_dense_topk_filtered(const void* queries, const void* items, int B, int N, int D, int dtype, int k,
                           int64_t id_offset, const rb_filter* filter, int64_t* out_ids, float* out_scores,
                           void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != RB_F16 && dtype != RB_BF16) return fail(RB_ERR_TYPE, "dense_topk_filtered: dtype must be f16 or bf16");
  if (filter == nullptr) return fail(RB_ERR_INVALID_ARG, "dense_topk_filtered: filter is null");
  FilterArgs f{};
  f.mode = filter->mode;
  f.terms = static_cast<const PredTerm*>(filter->terms);
  f.n_terms = filter->n_terms;
  f.attrs = filter->item_attrs;
  f.C = filter->n_clauses;
  f.A = filter->attr_width;
  f.bloom = filter->item_bloom;
  if (f.mode == RB_FILTER_BLOOM || f.mode == RB_FILTER_BLOOM_RECHECK) {
    f.slices = filter->item_bloom_slices;  // null: built into the workspace below
    if (f.slices != nullptr && (reinterpret_cast<uintptr_t>(f.slices) & 15u) != 0)
      return fail(RB_ERR_INVALID_ARG, "dense_topk_filtered: item_bloom_slices must be 16-byte aligned");
  }
  if (f.mode < RB_FILTER_NONE || f.mode > RB_FILTER_BLOOM_RECHECK)
    return fail(RB_ERR_INVALID_ARG, "dense_topk_filtered: unknown filter mode");
  if (f.mode != RB_FILTER_NONE && (f.terms == nullptr || f.n_terms == nullptr))
    return fail(RB_ERR_INVALID_ARG, "dense_topk_filtered: predicate terms missing");
  if ((f.mode == RB_FILTER_EXACT || f.mode == RB_FILTER_BLOOM_RECHECK) && (f.attrs == nullptr || f.C <= 0 || f.A <= 0))
    return fail(RB_ERR_INVALID_ARG, "dense_topk_filtered: exact attributes missing");
  if ((f.mode == RB_FILTER_BLOOM || f.mode == RB_FILTER_BLOOM_RECHECK) && f.bloom == nullptr)
    return fail(RB_ERR_INVALID_ARG, "dense_topk_filtered: bloom words missing");
  return dense_topk_impl(dtype == RB_BF16 ? 1 : 0, queries, nullptr, items, nullptr, B, N, D, k, id_offset, out_ids,
                         out_scores, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), &f);
}

int rb_dense_topk_scaled(const void* queries, const float* query_scales, const void* items, const float* item_scales,
                         int B, int N, int D, int dtype, int k, int64_t id_offset, int64_t* out_ids, float* out_scores,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != RB_E4M3) return fail(RB_ERR_TYPE, "dense_topk_scaled: dtype must be e4m3");
  if (query_scales != nullptr || item_scales != nullptr)
    return fail(RB_ERR_UNSUPPORTED, "dense_topk_scaled: e4m3 rows take no scales (pass null)");
  return dense_topk_impl(4, queries, query_scales, items, item_scales, B, N, D, k, id_offset,
                         out_ids, out_scores, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int rb_dense_topk_i8(const int8_t* query_codes, const float* query_scales, const int8_t* item_codes,
                     const float* item_scales, int B, int N, int D, int k, int64_t id_offset, int64_t* out_ids,
                     float* out_scores, void* workspace, size_t workspace_bytes, void* stream) {
  return dense_topk_impl(2, query_codes, query_scales, item_codes, item_scales, B, N, D, k, id_offset, out_ids,
                         out_scores, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int rb_dense_topk_launches(int B, int N, int D, int dtype, int k, int* n_launches) {
  if (n_launches == nullptr) return fail(RB_ERR_INVALID_ARG, "n_launches is null");
  (void)D;
  (void)dtype;
  if (B <= 0) {
    *n_launches = 0;
    return RB_OK;
  }
  if (N == 0) {
    *n_launches = 1;
    return RB_OK;
  }
  DensePlan pl;
  dense_plan(B, N, k, dense_row_bytes(D, dtype), pl, N, dense_scaled(dtype));
  if (pl.sample_stride == 0) {
    *n_launches = 2;  // full pass, merge
  } else if (dense_spec_applies(dtype == RB_I8 ? 2 : 0, nullptr) && dense_spec_rank(k, pl, 3) < k) {
    // sample pass, row select (both seeds), full pass, merge, then (B <= 128) check, second
    // pass, merge; or (B > 128) select, gather, compact pass, merge, scatter, second pass, merge
    *n_launches = B <= kSpecRows ? 7 : 11;
  } else {
    *n_launches = 4;  // sample pass, row select, full pass, merge
  }
  return RB_OK;
}

int rb_merge_topk_workspace_size(int W, int B, int kin, size_t* bytes) {
  if (bytes == nullptr || W < 1 || B < 0 || kin < 0) return fail(RB_ERR_INVALID_ARG, "merge_topk: bad arguments");
  *bytes = merge_shard_ws_bytes(W, B, kin);
  return RB_OK;
}

int rb_merge_topk(const int64_t* ids, const float* scores, int W, int B, int kin, int k, int64_t* out_ids,
                  float* out_scores, void* workspace, size_t workspace_bytes, void* stream) {
  if (W < 1 || B < 0 || kin < 0 || k < 1) return fail(RB_ERR_INVALID_ARG, "merge_topk: bad arguments");
  if (k > 1024) return fail(RB_ERR_UNSUPPORTED, "merge_topk: k > 1024");
  if (B == 0) return RB_OK;
  if (workspace == nullptr || workspace_bytes < merge_shard_ws_bytes(W, B, kin))
    return fail(RB_ERR_WORKSPACE, "merge_topk: workspace too small");
  return merge_shard_lists(ids, scores, W, B, kin, k, out_ids, out_scores, workspace,
                           static_cast<cudaStream_t>(stream));
}

int rb_set_profile_events(void* start_event, void* stop_event) {
  ProfileEvents& pe = profile_events();
  pe.start = static_cast<cudaEvent_t>(start_event);
  pe.stop = static_cast<cudaEvent_t>(stop_event);
  return RB_OK;
}

int rb_workspace_device_error(const void* workspace, size_t workspace_bytes, int* err_out) {
  if (workspace == nullptr || err_out == nullptr || workspace_bytes < 256)
    return fail(RB_ERR_INVALID_ARG, "workspace_device_error: bad arguments");
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, ws_err_word(const_cast<void*>(workspace), workspace_bytes), sizeof(int),
                             cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(RB_ERR_CUDA, cudaGetErrorString(e));
  *err_out = v;
  return RB_OK;
}

}  // extern "C"
