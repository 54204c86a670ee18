/*
 * retrieve_b200 C-ABI: the scoring-and-selection hot path of torchretrieve
 * (rmnigm/retrieve) as sm_100a CUDA kernels behind plain C entry points.
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are device pointers to contiguous row-major memory.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); every kernel
 *     runs on it and no entry point synchronises the host.
 *   - No entry point allocates memory. Scratch space comes from the caller
 *     through `workspace` / `workspace_bytes`, sized by the matching
 *     *_workspace_size query (which is host-only and allocation-free too).
 *   - Return value: RB_OK or one of the RB_ERR_* codes below; the message of
 *     the last failure on the calling thread is available from rb_last_error().
 *     RB_ERR_INVALID_ARG maps to Python ValueError, RB_ERR_TYPE to TypeError,
 *     everything else to RuntimeError (the reference's error convention,
 *     retrieve/src/retrieve/ops/triton/fused_masked_knn_topk.py:188-194).
 *   - Top-k outputs are (ids int64 [B, k], scores fp32 [B, k]) sorted by score
 *     descending, ties broken toward the lower item id; rows with fewer than k
 *     candidates end in id -1 / score -inf
 *     (retrieve/src/retrieve/functional.py:57-85, interfaces.py:69-73).
 */
#ifndef RETRIEVE_B200_H_
#define RETRIEVE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(RB_BUILD) && defined(__GNUC__)
#define RB_API __attribute__((visibility("default")))
#else
#define RB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define RB_OK 0
#define RB_ERR_INVALID_ARG 1
#define RB_ERR_TYPE 2
#define RB_ERR_UNSUPPORTED 3
#define RB_ERR_WORKSPACE 4
#define RB_ERR_CUDA 5
#define RB_ERR_DEVICE 6

/* element types */
#define RB_F16 0
#define RB_BF16 1
#define RB_I8 2
#define RB_F32 3
#define RB_E4M3 4

/* Message of the last failed call on this thread ("" if none). */
RB_API const char* rb_last_error(void);

/* ABI version of this library. */
RB_API int rb_abi_version(void);

/*
 * Dense fused scoring + top-k over a resident item table.
 *   queries [B, D] and items [N, D], both f16 or both bf16 (dtype), fp32
 *   accumulation on the tensor cores (tcgen05), no [B, N] intermediate.
 *   id_offset is added to every returned id (row-sharded corpora).
 * Replaces PostfilterKNN.score + masked_topk
 *   (retrieve/src/retrieve/modules/knn.py:62-76; the reference scores with
 *   torch.mm(q, E_t, out_dtype=float32) then torch.topk, functional.py:30-85).
 * Supported: D * 2 in {128, 256, 512} bytes, 1 <= k <= 1024, N < 2^31.
 */
RB_API int rb_dense_topk_workspace_size(int B, int N, int D, int dtype, int k, size_t* bytes);
RB_API int rb_dense_topk(const void* queries, const void* items, int B, int N, int D, int dtype, int k, int64_t id_offset,
                  int64_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Exact clause filter over items [N, C, A] int64 (-1 pad), reverse flags
 * [C] uint8, queries [B, C] int64 (-1 = inactive clause).
 * scores == NULL: out is [B, N] uint8 (bool) -> retrieve::clause_mask
 *   (retrieve/src/retrieve/ops/triton/clause_mask.py:270-283).
 * scores != NULL ([B, N] fp32): out is [B, N] fp32 with failing items at -inf
 *   -> retrieve::clause_mask_scores (clause_mask.py:286-303).
 * B <= 65535.
 */
RB_API int rb_clause_mask(const int64_t* item_attrs, int N, int C, int A, const uint8_t* is_reverse,
                          const int64_t* query_attrs, int B, const float* scores, void* out, void* stream);

/*
 * Clause filter + stream compaction -> retrieve::clause_compact
 * (retrieve/src/retrieve/ops/triton/clause_compact.py:174-196): out_ids [B, N]
 * int64 holds each row's passing ids in ascending order on [0, out_counts[b]),
 * the tail is left unwritten; out_counts [B] int64. B <= 65535.
 */
RB_API int rb_clause_compact_workspace_size(int B, int N, size_t* bytes);
RB_API int rb_clause_compact(const int64_t* item_attrs, int N, int C, int A, const uint8_t* is_reverse,
                             const int64_t* query_attrs, int B, int64_t* out_ids, int64_t* out_counts,
                             void* workspace, size_t workspace_bytes, void* stream);

/*
 * Single fp16 query [1, D] against the fp16 table items_t [D, N] -> out [N]
 * fp32, one fp32 FMA per k in order k = 0 .. D-1 -> retrieve::gemv_scores
 * (retrieve/src/retrieve/ops/triton/gemv_scores.py:19-43).
 */
RB_API int rb_gemv_scores(const void* query, const void* items_t, int D, int N, float* out, void* stream);

/*
 * Top-k over per-query candidates positive_indices [B, P] int64 bounded by
 * counts [B] int64.
 * kind 0 -> retrieve::fused_masked_knn_topk
 *   (retrieve/src/retrieve/ops/triton/fused_masked_knn_topk.py:289-310):
 *   fp32 dot of query [B, D] and item_embs [N, D] (each fp16 or fp32),
 *   output [B, k], non-finite winners id -1; 1 <= k <= 224.
 * kind 1 -> retrieve::oporp_1bit_match_topk_indirect
 *   (retrieve/src/retrieve/ops/triton/oporp_1bit_match_topk.py:276-292):
 *   score 64*W - 2*popcount(q ^ x) over int64 words (D = W), output
 *   [B, min(k, P)]; min(k, P) <= 224.
 * Ties go to the lower candidate index. Ids outside [0, N) are never scored.
 */
RB_API int rb_candidate_topk_workspace_size(int B, int P, size_t* bytes);
RB_API int rb_candidate_topk(int kind, const void* query, int query_dtype, const void* items, int item_dtype, int N,
                             int D, const int64_t* positive_indices, int P, const int64_t* counts, int B, int k,
                             int64_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes,
                             void* stream);

/*
 * Full-scan 1-bit Hamming top-k -> retrieve::oporp_1bit_match_topk_full
 * (retrieve/src/retrieve/ops/triton/oporp_1bit_match_topk.py:261-273):
 * query_bits [B, W], item_bits [N, W] int64, score 64*W - 2*popcount as fp32,
 * output [B, k] (ids = item rows), ties to the lower row. W even, <= 16;
 * k <= 1024.
 */
RB_API int rb_hamming_topk_workspace_size(int B, int N, int W, int k, size_t* bytes);
RB_API int rb_hamming_topk(const int64_t* query_bits, const int64_t* item_bits, int B, int N, int W, int k,
                           int64_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * Per-row symmetric int8 quantization of x [B, D] fp32 -> codes [B, D] int8,
 * scales [B] fp32 (retrieve/src/retrieve/indexing/quantize.py:9-18
 * `quantize_int8` as it evaluates on a CUDA tensor, bit for bit: the scale is
 * abs_max * fp32(1/127), as in silvertorch/ops/csrc/fork_search_cuda.cu:686).
 */
RB_API int rb_quantize_int8(const float* x, int B, int D, int8_t* codes, float* scales, void* stream);

/*
 * Per-tensor symmetric int8 quantization of x [N, D] fp32
 * (retrieve/src/retrieve/indexing/quantize.py:34-52 `quantize_int8_global` on CUDA
 * tensors): abs_max = max(max |x|, 1e-8) over the table (NaN propagates);
 * codes[i] = clamp(round_half_even(fp32(x[r] / abs_max) * 127), -128, 127) for
 * r = rows[i] (or r = i when rows is NULL; then n_rows is ignored and N rows are
 * written); a row index outside [0, N) writes zeros; *scale (device) =
 * abs_max * fp32(1/127). Workspace from rb_quantize_int8_global_workspace_size.
 */
RB_API int rb_quantize_int8_global_workspace_size(size_t* bytes);
RB_API int rb_quantize_int8_global(const float* x, int64_t N, int D, const int64_t* rows, int64_t n_rows,
                                   int8_t* codes, float* scale, void* workspace, size_t workspace_bytes,
                                   void* stream);

/*
 * SilverTorch's bundle-major bloom index on the device, replacing the CUDA impls of
 *   st::bloom_index_build(Tensor feature_ids, Tensor feature_offsets, Tensor feature_values,
 *                         float b_multiplier, int k, bool fast_build=False) -> (Tensor, Tensor)
 *   st::bloom_index_build_fixed(..., int bits_per_doc, int k, bool fast_build=False)
 * (silvertorch/ops/csrc/bloom_indexer.cpp:26-136; bloom_indexer_cuda.cu:291-340, 790-960).
 * feature_ids int32 [C]; feature_offsets int64 [N * C + 1] (CSR over (doc, feature));
 * feature_values int64 [n_values]. Two calls: rb_bloom_index_widths writes each
 * 2048-doc bundle's bits per doc (widths [ceil(N / 2048)]: bits_per_doc when > 0, else
 * trunc(fp64(max values of a doc in the bundle * k) * b_multiplier)) and their prefix
 * sums bundle_b_offsets [ceil(N / 2048) + 1]; the caller allocates a zeroed
 * bloom_index of bundle_b_offsets[last] * 32 words, and rb_bloom_index_fill sets, for
 * every value, bit 63 - d % 64 of word (bundle_b_offsets[d / 2048] + p) * 32 +
 * (d % 2048) / 64 at its first k distinct positions p = murmur3(feature id, value,
 * seed) % B over seeds 0, 1, ... (bloom_index_util.cuh:61-107, 185-208). 1 <= k <= 64.
 */
RB_API int rb_bloom_index_widths(const int64_t* feature_offsets, int64_t N, int C, int k, double b_multiplier,
                                 int64_t bits_per_doc, int64_t* widths, int64_t* bundle_b_offsets, void* stream);
RB_API int rb_bloom_index_fill(const int32_t* feature_ids, const int64_t* feature_offsets,
                               const int64_t* feature_values, int64_t n_values, int64_t N, int C, int k,
                               const int64_t* bundle_b_offsets, int64_t* bloom_index, int64_t index_words,
                               void* stream);

/*
 * Sign packing of values [M, D] fp32, D a multiple of 64, into words [M, D / 64]
 * int64: bit b of word w is set iff values[m, 64 w + b] > 0
 * (retrieve/src/retrieve/indexing/quantize.py:63-72 `_pack_signs_to_int64`, the last
 * step of the SimHash and Sign-OPORP projections).
 */
RB_API int rb_pack_signs(const float* values, int64_t M, int D, int64_t* out_words, void* stream);

/* Number of kernel launches one rb_dense_topk call with these sizes makes. */
RB_API int rb_dense_topk_launches(int B, int N, int D, int dtype, int k, int* n_launches);

/*
 * Merge of W per-shard top-k results into the global top-k: ids/scores are
 * [W, B, kin] (id -1 = empty slot, ids < 2^32), output [B, k] with the same
 * ordering and padding rules. This is the step after the all-gather of a
 * row-sharded corpus; the reference has no multi-GPU path (its harness merges
 * chunked top-k lists the same way, evaluation/bench/oracle.py:83-92).
 */
RB_API int rb_merge_topk_workspace_size(int W, int B, int kin, size_t* bytes);
RB_API int rb_merge_topk(const int64_t* ids, const float* scores, int W, int B, int kin, int k, int64_t* out_ids,
                         float* out_scores, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Profiling hook: records two caller-owned cudaEvent_t on the call's stream
 * around the dominant kernel of every later call made from this thread (the
 * dense scan's full-corpus pass; rb_st_search's scorer); pass NULL, NULL to
 * stop. Used by bench.py to time that kernel on the stream it runs on.
 */
RB_API int rb_set_profile_events(void* start_event, void* stop_event);

/*
 * rb_dense_topk without a caller workspace, for callers that cannot allocate
 * device memory on the call path: a host whose device memory is owned by
 * another allocator and fixed at start-up, or a foreign-language runtime with
 * no caching allocator, where a cudaMalloc per call would synchronise the
 * device. The scratch is one static device array of
 * rb_dense_topk_noalloc_scratch_bytes() bytes (32 MiB) that every GPU loading
 * this library keeps until the process exits; calls whose scratch need is
 * larger return RB_ERR_WORKSPACE. The first call on a device looks the array's
 * device address up (it may load the module): make it before any stream
 * capture. The stream must belong to the current device (else
 * RB_ERR_INVALID_ARG), and a device reset leaves the looked-up address stale.
 * All calls share the array: calls that overlap on the GPU race and must be
 * serialised. Same arguments, results, checks and error codes as rb_dense_topk
 * otherwise. This entry point has no counterpart in the reference.
 */
RB_API size_t rb_dense_topk_noalloc_scratch_bytes(void);
RB_API int rb_dense_topk_noalloc(const void* queries, const void* items, int B, int N, int D, int dtype, int k,
                                 int64_t id_offset, int64_t* out_ids, float* out_scores, void* stream);

/*
 * Attribute predicates for the filtered dense search. Per query up to
 * RB_MAX_TERMS terms "clause == value", each possibly negated (flags bit 3),
 * combined as AND over groups (flags bits 0-2) of OR over the group's terms.
 * This covers LiNR's exact clause filter (one group per active clause, negate
 * = clause_is_reverse; retrieve/src/retrieve/functional.py:173-185) and the
 * AND / OR / NOT expressions of SilverTorch's query DSL once put in
 * conjunctive form (silvertorch/silvertorch/ops/csrc/EXPRESSION_SYNTAX.md).
 * A term matches exactly when some value of the item's clause equals `value`
 * (item_attrs [N, n_clauses, attr_width] int64, -1 pads), or through the
 * item's 64-bit Bloom word when every bit of `bloom_mask` is set
 * (silvertorch bloom_index_search_cuda.cu:304-349 on a 64-bit-per-doc index).
 * Mode BLOOM_RECHECK requires both the Bloom and the exact predicate.
 */
#define RB_MAX_TERMS 8
#define RB_FILTER_NONE 0
#define RB_FILTER_EXACT 1
#define RB_FILTER_BLOOM 2
#define RB_FILTER_BLOOM_RECHECK 3
typedef struct {
  int64_t value;
  uint64_t bloom_mask;
  int32_t clause;
  int32_t flags;
} rb_pred_term;
typedef struct {
  int mode;
  const void* terms;       /* rb_pred_term [B, RB_MAX_TERMS] */
  const int32_t* n_terms;  /* [B]; 0 = every item passes */
  const int64_t* item_attrs;
  int n_clauses;
  int attr_width;
  const uint64_t* item_bloom;
  /* Optional (null: built into the workspace on every call): the same Bloom words bit-sliced by
   * rb_bloom_slices at build time (the scan tests 32 items per term with one AND). */
  const uint32_t* item_bloom_slices;
} rb_filter;

/*
 * Dense fused scoring + top-k with an attribute predicate folded into the scan
 * (LiNR V1 with its filter, retrieve/src/retrieve/modules/linr.py:75-79, and the
 * bloom-filtered scan): items failing the predicate never enter the top-k; rows
 * with fewer than k passing items end in -1 / -inf. Other arguments and limits
 * as rb_dense_topk. Workspace: rb_dense_topk_filtered_workspace_size, which for
 * the Bloom modes adds room for the words bit-sliced (8 bytes an item), so that
 * the scans test a 32-item chunk per term with one AND; a workspace of
 * rb_dense_topk_workspace_size bytes still works, testing item by item.
 */
RB_API int rb_dense_topk_filtered_workspace_size(int B, int N, int D, int dtype, int k, int mode, size_t* bytes);
RB_API int rb_dense_topk_filtered(const void* queries, const void* items, int B, int N, int D, int dtype, int k,
                                  int64_t id_offset, const rb_filter* filter, int64_t* out_ids, float* out_scores,
                                  void* workspace, size_t workspace_bytes, void* stream);

/*
 * Per-item 64-bit Bloom words from item_attrs [N, C, A] int64 (-1 pads; the
 * clause index is the feature id): bit p of word n is set iff p is one of the
 * first k distinct murmur_hash3_2x64(clause, value, seed) % 64 over
 * seed = 0, 1, ... for some (clause, value) of item n
 * (silvertorch bloom_index_util.cuh:61-107, 185-208). Build time.
 */
RB_API int rb_bloom_build(const int64_t* item_attrs, int N, int C, int A, int k, uint64_t* out_words, void* stream);

/*
 * The per-item Bloom words bit-sliced for the filtered scans, built once with the index (no
 * counterpart in the reference, whose Bloom index is tested word by word): per 32-item chunk
 * 64 uint32 words, word p holding bit p of the chunk's 32 items, whole 128-item tiles (zero
 * words past N): rb_bloom_slices_bytes(N) bytes. Given to rb_dense_topk_filtered as
 * rb_filter.item_bloom_slices, they save the per-call build (0.25 ms at 10M items).
 */
RB_API int rb_bloom_slices_bytes(int64_t N, size_t* bytes);
RB_API int rb_bloom_slices(const uint64_t* item_bloom, int64_t N, uint32_t* out_slices, void* stream);

/*
 * Int8 scoring + top-k (tensor-core int8 x int8 -> int32 dots, kind::i8):
 * query_codes [B, D] and item_codes [N, D] int8, per-query and per-item fp32
 * scales; score = (fp32(dot) * query_scale) * item_scale in that order
 * (the dequant of retrieve/src/retrieve/ops/official/adapter.py:338-367 and
 * silvertorch fork_search_cuda.cu:585-591; with one global item scale this is
 * SilverTorch's int32 scoring path over every item). D in {128, 256, 512};
 * k <= 1024. A null scale array means unit scales: the score is then the raw
 * int32 dot as fp32 (exact; with +-1 codes from rb_bits_to_pm1 it is the
 * 1-bit match score 64 W - 2 hamming). Workspace as rb_dense_topk_workspace_size.
 */
RB_API int rb_dense_topk_i8(const int8_t* query_codes, const float* query_scales, const int8_t* item_codes,
                            const float* item_scales, int B, int N, int D, int k, int64_t id_offset,
                            int64_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes,
                            void* stream);

/*
 * Expands 1-bit codes [N, W] int64 (bit b of word w = coordinate 64 w + b, LSB
 * first; retrieve/src/retrieve/indexing/quantize.py:63-72) into a +-1 int8
 * table [N, 64 W]: +1 where the bit is set. The dot of two such rows is
 * 64 W - 2 popcount(q ^ x), the score of oporp_1bit_match_topk
 * (retrieve/src/retrieve/ops/reference/oporp_1bit_match_topk.py:9-41), so
 * rb_dense_topk_i8 with null scales ranks 1-bit codes on the tensor cores.
 * Index-build time (8x the packed size); queries per batch.
 */
RB_API int rb_bits_to_pm1(const int64_t* bits, int N, int W, int8_t* out, void* stream);

/*
 * Dense top-k over fp8 e4m3 rows (kind::f8f6f4, fp32 accumulation, score = the
 * accumulator). dtype must be RB_E4M3 and both scale arrays null (reserved);
 * rows of 128 / 256 / 512 bytes; k <= 1024. With +-1 codes
 * (rb_bits_to_pm1_e4m3) every partial sum is an integer of at most 512 in
 * magnitude, so the scores are the exact 1-bit match scores 64 W - 2 hamming.
 * Workspace as rb_dense_topk_workspace_size with the same dtype.
 */
RB_API int rb_dense_topk_scaled(const void* queries, const float* query_scales, const void* items,
                                const float* item_scales, int B, int N, int D, int dtype, int k, int64_t id_offset,
                                int64_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes,
                                void* stream);

/* rb_bits_to_pm1 with fp8 e4m3 output (+1.0 = 0x38, -1.0 = 0xb8). */
RB_API int rb_bits_to_pm1_e4m3(const int64_t* bits, int N, int W, uint8_t* out, void* stream);

/*
 * Reads (synchronously) the device error word a scan kernel leaves in
 * `workspace` (0 = none; non-zero = a bounded wait ran out). Test / debug aid.
 */
RB_API int rb_workspace_device_error(const void* workspace, size_t workspace_bytes, int* err_out);

/*
 * Test aid for the bounded waits: launches one CTA whose producer, MMA and
 * epilogue roles each wait, through the scan kernels' own bounded wait, on an
 * mbarrier that nothing completes, with a limit of limit_ns (1 us .. 2 s) in
 * place of the kernels' 2 s. The first role to give up writes its timeout code
 * (1 producer, 2 MMA, 3 epilogue) to the error word at the end of `workspace`
 * (read it with rb_workspace_device_error) and the kernel returns. No
 * counterpart in the reference.
 */
RB_API int rb_wait_probe(int64_t limit_ns, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Row-sharded search with one threshold for all shards (no counterpart in the
 * reference, which is single-GPU). A shard of N of the n_total corpus rows:
 *
 *   rb_dense_seed_sample writes out_vals [B, m] fp32 (1 <= m <= k): per query,
 *   m tile maxima (max of 128 consecutive items) from this shard's sampling
 *   pass, all at or above the shard's own m-th largest tile max (-inf where
 *   the shard sampled fewer). The caller gathers every shard's [B, m] into a
 *   [W, B, m] stack (one all-gather) and passes it to
 *
 *   rb_dense_topk_seeded: as rb_dense_topk on the shard, with the full pass
 *   seeded by the k-th largest value of the union of the W samples. Any k of
 *   those values come from k distinct chunks, so that is a lower bound on the
 *   k-th best score of the whole corpus (whatever m is): every item of the
 *   global top-k is kept by its shard and the per-shard results merge
 *   (rb_merge_pairs / rb_merge_topk) to the exact global top-k, while each
 *   shard appends only about 1/W of the candidates a shard-local seed lets
 *   through. m about 2k/W keeps the bound as tight as m = k unless one shard
 *   holds more than m of the global top chunks. A shard may return fewer than
 *   k real entries (-1 / -inf pads).
 *
 * Both use the workspace of rb_dense_topk_workspace_size(B, N, ...); the same
 * n_total must be given to both calls. fp16 / bf16 only.
 *
 * With out_pairs not null, rb_dense_topk_seeded writes its [B, k] result there
 * instead of out_ids / out_scores (which may then be null) as 8-byte pairs: the
 * fp32 score's bits in the low 32 bits, the uint32 global id in the high 32
 * bits (padding: -inf and 0xffffffff); global ids must stay below 2^32 - 1.
 * One all-gather of the pairs gives the [W, B, k] stack that rb_merge_pairs
 * reduces to the global top-k (ids int64, -1 / -inf pads).
 */
RB_API int rb_dense_seed_sample(const void* queries, const void* items, int B, int N, int D, int dtype, int k,
                                int m, int64_t n_total, float* out_vals, void* workspace, size_t workspace_bytes,
                                void* stream);
RB_API int rb_dense_topk_seeded(const void* queries, const void* items, int B, int N, int D, int dtype, int k,
                                int64_t id_offset, int64_t n_total, const float* seed_vals, int W, int m,
                                int64_t* out_ids, float* out_scores, uint64_t* out_pairs, void* workspace,
                                size_t workspace_bytes, void* stream);
RB_API int rb_merge_pairs(const uint64_t* pairs, int W, int B, int kin, int k, int64_t* out_ids, float* out_scores,
                          void* stream);

/*
 * The all-gather of the row-sharded search through the peers' memory on one
 * node, in place of NCCL's (no counterpart in the reference: it is single-GPU).
 * Every rank allocates one exchange buffer of rb_peer_buffer_bytes(W,
 * slot_bytes) with rb_ipc_alloc, passes the 64-byte IPC handle to its peers
 * (any host channel) and maps theirs with rb_ipc_open. rb_peer_allgather then
 * pushes this rank's `bytes` (a multiple of 16, at most slot_bytes) into every
 * rank's buffer with plain peer stores, raises this rank's flag there, waits
 * (bounded: 2 s) until every rank's flag for the step is up in its own buffer
 * and writes the [W, bytes] stack, in rank order, to `out` (device). `bases`
 * is a host array of the W buffers (index = rank; this rank's own allocation
 * at `rank`); `step` (int64), `done` (int) are this rank's device counters,
 * zeroed once, and `err` its error word (5 = a peer did not arrive in time).
 * Every rank calls it the same number of times, on its own GPU; the step
 * counter lives on the device, so a captured graph replays it. No multicast.
 */
RB_API int rb_ipc_alloc(size_t bytes, void** ptr, void* handle);
RB_API int rb_ipc_open(const void* handle, void** ptr);
RB_API int rb_ipc_close(void* ptr);
RB_API int rb_ipc_free(void* ptr);
RB_API size_t rb_peer_buffer_bytes(int W, int64_t slot_bytes);
RB_API int rb_peer_allgather(void* const* bases, int W, int rank, int64_t slot_bytes, const void* src, int64_t bytes,
                             int64_t* step, int* done, int* err, void* out, void* stream);

/*
 * The filter of one st::search call: at most one of the three groups is set (NULL
 * pointers for the others), or pass a NULL rb_st_filter* for none.
 *   filtering_bit_mask [B, mask_words] int64 over sorted positions, high bit first
 *     (position d at bit 63 - d % 64 of word d / 64);
 *   the exact clauses (silvertorch/ops/csrc/fork_filters.cuh:15-41): item_clause_attrs
 *     int32 [attr_rows, attr_docs >= N] (clause c in rows clause_slots[c] ..
 *     clause_slots[c + 1], each doc's values sorted descending, -1 pads), clause_slots
 *     int64 [n_clauses + 1], clause_is_reverse bool [n_clauses], query_clause_attrs
 *     int32 [B, n_clauses] (-1: clause inactive);
 *   SilverTorch's bloom (bloom_index_search_cuda.cu:304-349, 469-544): bloom_index int64
 *     [bloom_words] bundle-major, bundle_b_offsets int64 [n_bundles + 1], plans int64
 *     [plan_words] (per slot the parser's eight byte offsets, then its data;
 *     retrieve/src/retrieve/ops/official/adapter.py:212-236), plan_count slots,
 *     max_stack_size (<= 16), query_plan_index int64 [B] or NULL (row b: plan b),
 *     bloom_k distinct positions (<= 10) among hash_k stored hashes a term.
 * With the bloom and its exact recheck (both in the reference op) pass the exact
 * clauses only: the bloom has no false negatives, so the result is the same.
 */
typedef struct rb_st_filter {
  const int64_t* filtering_bit_mask;
  int64_t mask_words;
  const int32_t* item_clause_attrs;
  int64_t attr_rows;
  int64_t attr_docs;
  const int64_t* clause_slots;
  const uint8_t* clause_is_reverse;
  const int32_t* query_clause_attrs;
  int n_clauses;
  const int64_t* bloom_index;
  int64_t bloom_words;
  const int64_t* bundle_b_offsets;
  int64_t n_bundles;
  const int64_t* plans;
  int64_t plan_words;
  int plan_count;
  int max_stack_size;
  const int64_t* query_plan_index;
  int bloom_k;
  int hash_k;
} rb_st_filter;

/*
 * SilverTorch's IVF probe search, replacing the CUDA impl of
 *   st::search(Tensor query, Tensor probe_ids, Tensor cluster_offsets, Tensor cluster_sizes,
 *              Tensor item_codes, Tensor sort_perm, Tensor global_scale, int k,
 *              int max_tensor_size_per_row, int divisor_for_int8=-1,
 *              Tensor? filtering_bit_mask=None, ...) -> (Tensor, Tensor)
 * (silvertorch/ops/csrc/fork_search.cpp:14-41; fork_search_cuda.cu:1256-1524).
 *   query [B, D] fp32; probe_ids [B, P] int64 cluster ids; cluster_offsets
 *   [n_lists + 1] int64; cluster_sizes [n_lists] int64; item_codes [N, D] int8,
 *   cluster-sorted; sort_perm [N] int64 (sorted position -> item id);
 *   global_scale: one fp32 on the device; divisor_for_int8 -1 (rank on the int32
 *   dot) or a positive divisor (rank on fp16(dot / divisor)); filter: see rb_st_filter.
 * Output (ids int64 [B, k], scores fp32 [B, k]): the k best probed positions by
 * raw score, ties to the reference scorer's lower slot, id = sort_perm[pos],
 * score = (fp32(dot) * q_scale) * global_scale, or
 * raw * ((q_scale * divisor) * global_scale); -1 / -inf past the candidates.
 * Limits: D <= 1024, P <= 2048, B <= 65535, min(k, round_up(width, 32)) <= 1024.
 * Workspace from rb_st_search_workspace_size.
 */
RB_API int rb_st_search_workspace_size(int B, int D, int P, int k, int max_tensor_size_per_row, size_t* bytes);
RB_API int rb_st_search(const float* query, int B, int D, const int64_t* probe_ids, int P,
                        const int64_t* cluster_offsets, const int64_t* cluster_sizes, int64_t n_lists,
                        const int8_t* item_codes, int64_t N, const int64_t* sort_perm, const float* global_scale, int k,
                        int max_tensor_size_per_row, int divisor_for_int8, const rb_st_filter* filter,
                        int64_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes,
                        void* stream);

/*
 * The same search, grouped by cluster: every (row, probe) pair is filed under its
 * cluster, and each cluster is read once per group of up to 64 probing rows
 * (staged in shared memory) instead of once per probing row. Same arguments,
 * results and limits as rb_st_search, with P <= 1024; workspace from
 * rb_st_search_grouped_workspace_size (it also depends on n_lists).
 */
RB_API int rb_st_search_grouped_workspace_size(int B, int D, int P, int64_t n_lists, int k,
                                               int max_tensor_size_per_row, size_t* bytes);
RB_API int rb_st_search_grouped(const float* query, int B, int D, const int64_t* probe_ids, int P,
                                const int64_t* cluster_offsets, const int64_t* cluster_sizes, int64_t n_lists,
                                const int8_t* item_codes, int64_t N, const int64_t* sort_perm,
                                const float* global_scale, int k, int max_tensor_size_per_row, int divisor_for_int8,
                                const rb_st_filter* filter, int64_t* out_ids, float* out_scores, void* workspace,
                                size_t workspace_bytes, void* stream);

/*
 * The same search over several GPUs, each holding the rows [pos_lo, pos_hi) of the sorted
 * table (whole clusters; item_codes = those rows): rb_st_search_shard scores the probed
 * positions in the window, keeping the global slot layout (the probe tables cluster_offsets /
 * cluster_sizes and the filter are the whole table's), and writes its best min(k, width)
 * as packed pairs out_pairs [B, min(k, width)]: raw score bits (fp32 of the int32 dot, or of
 * the fp16 path's value) in the low 32 bits, the slot in the high 32 (padding -inf /
 * 0xffffffff; workspace from rb_st_search_workspace_size). The pairs of all ranks merge with
 * rb_merge_pairs (raw descending, slot ascending: the single-GPU tie order) into slots /
 * raw [B, kin], and rb_st_search_finish maps each slot to its position through the whole
 * table's layout, then to sort_perm and the dequantized score, padding to k. The result
 * equals rb_st_search's on the whole table, ties included.
 */
RB_API int rb_st_search_shard(const float* query, int B, int D, const int64_t* probe_ids, int P,
                              const int64_t* cluster_offsets, const int64_t* cluster_sizes, int64_t n_lists,
                              int64_t N, int64_t pos_lo, int64_t pos_hi, const int8_t* item_codes, int k,
                              int max_tensor_size_per_row, int divisor_for_int8, const rb_st_filter* filter,
                              uint64_t* out_pairs, void* workspace, size_t workspace_bytes, void* stream);
RB_API int rb_st_search_finish_workspace_size(int B, int D, int P, size_t* bytes);
RB_API int rb_st_search_finish(const float* query, int B, int D, const int64_t* probe_ids, int P,
                               const int64_t* cluster_offsets, const int64_t* cluster_sizes, int64_t n_lists,
                               int64_t N, const int64_t* sort_perm, const float* global_scale, int k,
                               int max_tensor_size_per_row, int divisor_for_int8, const int64_t* slots,
                               const float* raw, int kin, int64_t* out_ids, float* out_scores, void* workspace,
                               size_t workspace_bytes, void* stream);

/*
 * The upstream-shaped raw scorer on int8 codes, replacing the CUDA impl of
 *   st::fused_kmean_ann(Tensor cluster_offsets, Tensor cluster_ids, Tensor cluster_length,
 *                       Tensor embeddings, Tensor queries, int max_tensor_size_per_row,
 *                       Tensor? filtering_bit_mask=None, int invalid_index_value=-1,
 *                       int divisor_for_int8=-1, ...) -> (Tensor, Tensor)
 * (silvertorch/ops/csrc/fused_kmean_ann.cpp:86-228 for the CPU form; fused_kmean_ann_cuda.cu
 * :2126-2262). cluster_ids / cluster_length [B, P] int64 (the probed clusters and their
 * lengths), embeddings [N, D] and queries [B, D] of one dtype: RB_I8, or RB_F32 / RB_F16 /
 * RB_BF16, for which out_raw has the embeddings' type and holds the CUDA scorer's fused
 * multiply-add chains (blocks of 256 or 384 bytes, fp16 / bf16 in even / odd pairs; D a
 * multiple of 16 bytes; pads -FLT_MAX / -65504 / bf16 0xff7f; divisor and per-doc scale unused).
 * Output [B, round_up(width, 32)]: in
 * the CUDA scorer's slot order (warp-aligned prefixes, then remainders), out_raw holds the
 * int32 dot (divisor -1) or fp16(fp32(dot) / divisor), out_idx the int32 position; empty,
 * filtered (filtering_bit_mask [mask_rows, mask_words], high bit first) and padding slots
 * hold INT32_MIN / -65504 and invalid_index_value. filtering_bit_index (int64 [B] or NULL)
 * makes row b read mask row filtering_bit_index[b] (an index outside [0, mask_rows) filters
 * the whole row out); without it mask_rows >= B. per_embedding_scale (fp16 bits [N] or NULL)
 * replaces the divisor by a per-doc one: fp16 raw fp16(fp32(fp16(dot)) / fp32(scale[doc])),
 * the CUDA scorer's order (index_mm_helpers.cuh:49-53). Workspace from
 * rb_st_fused_kmean_ann_workspace_size.
 */
RB_API int rb_st_fused_kmean_ann_workspace_size(int B, int P, int max_tensor_size_per_row, size_t* bytes);
RB_API int rb_st_fused_kmean_ann(const int64_t* cluster_offsets, int64_t n_lists, const int64_t* cluster_ids,
                                 const int64_t* cluster_length, int P, const void* embeddings, int64_t N,
                                 const void* queries, int dtype, int B, int D, int max_tensor_size_per_row,
                                 const int64_t* filtering_bit_mask, int64_t mask_rows, int64_t mask_words,
                                 const int64_t* filtering_bit_index, const uint16_t* per_embedding_scale,
                                 int invalid_index_value, int divisor_for_int8, void* out_raw, int32_t* out_idx,
                                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * st::fused_kmean_ann_with_partial_masks on int8 codes (schema
 * silvertorch/ops/csrc/fused_kmean_ann.cpp:416-437; CUDA fused_kmean_ann_cuda.cu:661-845):
 * rb_st_fused_kmean_ann with the bloom filter of the probed clusters only, the triple of
 * rb_st_bloom_partial_search: probe j of row b keeps the i-th doc of its range when bit
 * first_item_offset_in_column[b P + j] + i of column_results from word
 * column_counts_cumsum[b P + j - 1] on (word 0 for the first range) is set, high bit first.
 * n_column_results words are readable; a bit past them drops the doc. The triple covers
 * mask_rows x P ranges; filtering_bit_index (int64 [B] or NULL) makes row b read the ranges of
 * mask row filtering_bit_index[b] (outside [0, mask_rows): the whole row filtered out), else
 * mask_rows >= B. per_embedding_scale as in rb_st_fused_kmean_ann.
 */
RB_API int rb_st_fused_kmean_ann_with_partial_masks(
    const int64_t* cluster_offsets, int64_t n_lists, const int64_t* cluster_ids, const int64_t* cluster_length, int P,
    const void* embeddings, int64_t N, const void* queries, int dtype, int B, int D, int max_tensor_size_per_row,
    const int32_t* column_counts_cumsum, const int8_t* first_item_offset_in_column, const int64_t* column_results,
    int64_t n_column_results, int64_t mask_rows, const int64_t* filtering_bit_index,
    const uint16_t* per_embedding_scale, int invalid_index_value, int divisor_for_int8, void* out_raw,
    int32_t* out_idx, void* workspace, size_t workspace_bytes, void* stream);

/*
 * SilverTorch's bloom searches over the bundle-major index (layout of rb_bloom_index_fill), on
 * prepared plans (the blob st::search reads: 8 int64 offsets per plan slot, then the parser's
 * bytes; max_stack_size <= 16, 1 <= k <= 10):
 *
 * rb_st_bloom_search replaces st::bloom_index_search_batch(_prepared)
 * (silvertorch/ops/csrc/bloom_index_search.cpp:550-588; bloom_index_search_cuda.cu:1504-1640,
 * 1832-1859): plan q over every 64-doc column, out int64 [plan_count, n_bundles * 32] (doc
 * 64 c + i at bit 63 - i of word c) or, with return_bool_mask, uint8 0 / 1
 * [plan_count, n_bundles * 2048].
 *
 * rb_st_bloom_column_info replaces st::generate_column_info_for_clusters
 * (bloom_index_search.cpp:494-538): per range (start, length), int32 column count
 * ceil((length + start % 64) / 64) (0 when length <= 0), int32 first column start / 64,
 * int8 start % 64; with out_column_counts_cumsum not null also the inclusive int32 cumsum.
 *
 * rb_st_bloom_partial_search replaces the words of
 * st::bloom_index_search_batch_return_partial_response(_prepared) (bloom_index_search.cpp
 * :244-374; bloom_index_search_cuda.cu:1780-1944): over the B x P ranges of
 * rb_st_bloom_column_info, the words of each range's columns in order, row b running plan
 * query_plan_index[b] (or b); out [max_columns] int64, zero past the total.
 */
RB_API int rb_st_bloom_search(const int64_t* bloom_index, int64_t index_words, const int64_t* bundle_b_offsets,
                              int64_t n_bundles, const int64_t* plans, int64_t plan_words, int plan_count,
                              int max_stack_size, int k, int hash_k, int return_bool_mask, void* out, void* stream);
RB_API int rb_st_bloom_column_info(const int64_t* selected_cluster_offsets, const int64_t* selected_cluster_lengths,
                                   int64_t n, int32_t* out_column_counts, int32_t* out_start_column_ids,
                                   int8_t* out_first_item_offsets, int32_t* out_column_counts_cumsum, void* stream);
RB_API int rb_st_bloom_partial_search(const int64_t* bloom_index, int64_t index_words,
                                      const int64_t* bundle_b_offsets, int64_t n_bundles, const int64_t* plans,
                                      int64_t plan_words, int plan_count, int max_stack_size,
                                      const int64_t* query_plan_index, int B, int P,
                                      const int32_t* column_counts_cumsum, const int32_t* start_column_ids, int k,
                                      int hash_k, int64_t* out_column_mask_response, int64_t max_columns,
                                      void* stream);

/*
 * st::is_topk(Tensor scores, Tensor ks, Tensor(a!) is_topk_output, bool largest=True)
 * (silvertorch/ops/csrc/is_topk.cpp:84-90; CUDA is_topk_cuda.cu:83-149): for each row b of
 * scores [B, n] (dtype RB_F32, RB_F16 or RB_BF16) the value kth at position
 * clamp(ks[b] - 1, 0, n - 1) of the row sorted descending (ascending when largest is 0; NaN
 * sorts as the largest value), then out[b, j] = scores[b, j] >= kth (<= when smallest),
 * compared in fp32, as 1 / 0 in the scores' dtype. ks: int64 [B] on the device. n < 2^32.
 */
RB_API int rb_st_is_topk(const void* scores, int dtype, int64_t B, int64_t n, const int64_t* ks, int largest,
                         void* out, void* stream);

/*
 * st::take_top_k_and_gather_from_main_and_fresh (silvertorch/ops/csrc/
 * fresh_index_post_processing.cpp:226-286), in two calls:
 *
 * rb_st_fresh_topk: per row b the top k' = min(k, mf + mm) of the fresh scores [B, mf] followed
 * by the main scores [B, mm] (dtype RB_F32 / RB_F16 / RB_BF16), largest first with NaN the
 * largest and ties to the lower merged column: out_scores [B, k'] (the scores' dtype), out_idx
 * [B, k'] int64 merged columns (fresh j -> j, main j -> mf + j), out_is_fresh [B, k'] 0 / 1 bytes.
 * mf + mm <= 4096.
 *
 * rb_st_fresh_gather: for the [B, k_out] merged columns top_idx, the data row of each winner
 * copied to out [B * k_out, row_elems] (elem_bytes 1, 2, 4 or 8 a value): fresh_data
 * [fresh_rows, row_elems] at fresh_indices[b, col] for col < mf, main_data at
 * main_indices[b, col - mf] otherwise (indices int32 or int64, [B, mf] and [B, mm]); an index
 * outside its table reads row 0.
 */
RB_API int rb_st_fresh_topk(const void* fresh_scores, int64_t mf, const void* main_scores, int64_t mm, int dtype,
                            int64_t B, int k, void* out_scores, int64_t* out_idx, uint8_t* out_is_fresh,
                            void* stream);
RB_API int rb_st_fresh_gather(const int64_t* top_idx, int64_t B, int k_out, int64_t mf, int64_t mm,
                              const void* fresh_indices, const void* main_indices, int indices_are_int64,
                              const void* fresh_data, int64_t fresh_rows, const void* main_data, int64_t main_rows,
                              int64_t row_elems, int elem_bytes, void* out, void* stream);

/*
 * The centroid update of the IVF build's k-means, replacing KMeans._cluster_sums
 * (retrieve/src/retrieve/indexing/kmeans.py:98-119, an fp64 one-hot GEMM per row chunk):
 * out_sums [n_lists, D] fp64 = per cluster the sum of its rows of embs [N, D] (dtype RB_F32,
 * RB_F16 or RB_BF16), out_counts [n_lists] int64 = its rows, for assignments [N] int64 (rows
 * assigned outside [0, n_lists) are left out). Each cluster's rows are added in increasing row
 * order in fp64 after a stable counting sort: bit-for-bit reproducible, equal to the reference's
 * sums whenever the fp64 additions are exact. 1 <= n_lists <= 2^24. Workspace from
 * rb_kmeans_cluster_sums_workspace_size.
 */
RB_API int rb_kmeans_cluster_sums_workspace_size(int64_t N, int64_t n_lists, size_t* bytes);
RB_API int rb_kmeans_cluster_sums(const void* embs, int dtype, int64_t N, int D, const int64_t* assignments,
                                  int64_t n_lists, double* out_sums, int64_t* out_counts, void* workspace,
                                  size_t workspace_bytes, void* stream);

/*
 * SilverTorch's expression parser on the host, replacing
 *   st::parse_expression_query_batch(str[] expressions, Tensor silvertorch_ks, int bloom_hash_k,
 *                                    bool return_query_plan=True, int max_sub_queries=5)
 * (silvertorch/ops/csrc/expression_query_parser.cpp:395-430; encoding
 * bloom_index_util.cpp:27-127): n_expressions strings (bytes and lengths, no terminator
 * needed) compiled to the parser's plan bytes, byte-identical to the reference's. Writes
 * *out_data_bytes and *out_max_stack; with out_data and out_offsets both NULL that is all
 * (a size query), else out_data (data_capacity >= *out_data_bytes bytes) receives the plan
 * bytes and out_offsets the 8 byte offsets of each plan. A malformed expression returns
 * RB_ERR_INVALID_ARG with the position in rb_last_error(). 1 <= bloom_hash_k <= 2^20.
 */
RB_API int rb_st_parse_expression_batch(const char* const* expressions, const int64_t* lengths, int n_expressions,
                                        int64_t bloom_hash_k, int64_t max_sub_queries, int8_t* out_data,
                                        int64_t data_capacity, int64_t* out_offsets, int64_t* out_data_bytes,
                                        int64_t* out_max_stack);

/*
 * st::probe_prep(Tensor query, Tensor probe_ids, Tensor cluster_offsets, Tensor cluster_sizes)
 *   -> (codes int8 [B, D], scales fp32 [B], cluster_ids int64 [B, P],
 *       cluster_length int64 [B, P], cluster_offsets int64 [B, P], warps int32 [B * P],
 *       warp_rounded_length_cumsum int32 [B, P] (per row), remaining_length_cumsum
 *       int32 [B * P] (global), warp_size_cumsum int32 [B * P] (global))
 * (silvertorch/ops/csrc/fork_search.cpp:43-49; fork_search_cuda.cu:1529-1546; the
 * layout the reference checks at retrieve/tests/parity/test_official.py:676-697).
 */
RB_API int rb_st_probe_prep(const float* query, int B, int D, const int64_t* probe_ids, int P,
                            const int64_t* cluster_offsets, const int64_t* cluster_sizes, int64_t n_lists,
                            int8_t* out_codes, float* out_scales, int64_t* out_cluster_ids,
                            int64_t* out_cluster_length, int64_t* out_cluster_offsets, int32_t* out_warps,
                            int32_t* out_rounded_cumsum, int32_t* out_remaining_cumsum, int32_t* out_warp_cumsum,
                            void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RETRIEVE_B200_H_ */
