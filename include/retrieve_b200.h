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
 * Supported: D * 2 in {128, 256} bytes, 1 <= k <= 256, N < 2^31.
 */
RB_API int rb_dense_topk_workspace_size(int B, int N, int D, int dtype, int k, size_t* bytes);
RB_API int rb_dense_topk(const void* queries, const void* items, int B, int N, int D, int dtype, int k, int64_t id_offset,
                  int64_t* out_ids, float* out_scores, void* workspace, size_t workspace_bytes, void* stream);

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
 * around the dominant kernel (the full-corpus scan) of every later call made
 * from this thread; pass NULL, NULL to stop. Used by bench.py to time that
 * kernel on the stream it runs on.
 */
RB_API int rb_set_profile_events(void* start_event, void* stop_event);

/*
 * rb_dense_topk without a caller workspace, for callers that cannot allocate
 * device memory on the call path (a host recording the search into a CUDA
 * graph, where cudaMalloc is not allowed during capture, or a host whose device
 * memory is fixed at start-up by another allocator). The scratch is one static
 * device array of rb_dense_topk_noalloc_scratch_bytes() bytes (32 MiB) that
 * every GPU loading this library keeps until the process exits; calls whose
 * scratch need is larger return RB_ERR_WORKSPACE. The first call on a device
 * looks the array's device address up (it may load the module): make it before
 * any stream capture. All calls share the array: calls that overlap on the GPU
 * race and must be serialised. Same arguments, results and limits as
 * rb_dense_topk otherwise. This entry point has no counterpart in the reference.
 */
RB_API size_t rb_dense_topk_noalloc_scratch_bytes(void);
RB_API int rb_dense_topk_noalloc(const void* queries, const void* items, int B, int N, int D, int dtype, int k,
                                 int64_t id_offset, int64_t* out_ids, float* out_scores, void* stream);

/*
 * Reads (synchronously) the device error word a scan kernel leaves in
 * `workspace` (0 = none; non-zero = a bounded wait ran out). Test / debug aid.
 */
RB_API int rb_workspace_device_error(const void* workspace, size_t workspace_bytes, int* err_out);

#ifdef __cplusplus
}
#endif

#endif /* RETRIEVE_B200_H_ */
