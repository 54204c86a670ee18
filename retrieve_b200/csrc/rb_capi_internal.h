// Host-side declarations shared by the .cu files behind the C-ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "retrieve_b200.h"
#include "rb_common.cuh"

namespace rb {

// Device ordinals whose per-device lookups (SM count, CTA-pair occupancy) are cached.
constexpr int kMaxCachedDevices = 64;

void set_last_error(const char* msg);

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// How one dense top-k call is cut into scan passes (see dense_scan_sm100.cu).
struct DensePlan {
  bool two_sm;   // CTA-pair kernel (M = 256 per group) or the 1-SM kernel (M = 128)
  int ng;        // query groups per CTA (pair)
  int n_qsg;     // query super-groups (ng groups each)
  int n_splits;  // item splits per super-group
  int n_lists;   // candidate lists per query (splits x column halves)
  int cap;       // candidate-list capacity per (query, split)
  int tiles;     // 128-item tiles in the corpus
  int sample_stride;  // 0: no sampling pass; else the tile stride of the sample
};

void dense_plan(int B, int N, int k, int row_bytes, DensePlan& pl, int64_t n_total = 0, bool scaled = false);
// Rows a speculative search's compact second pass takes (one 128-row query group), and the
// workspace its buffers need past the seeds (capi.cu's SpecWs).
constexpr int kSpecRows = 128;
size_t dense_spec_ws_bytes(int k);
size_t dense_workspace_bytes(int B, int N, int k, int row_bytes, bool scaled = false);
// Element types with the per-query / per-item dequant in the epilogue.
inline bool dense_scaled(int dtype) { return dtype == RB_I8 || dtype == RB_E4M3; }
// Bytes of one item row for a dtype code (RB_I8: D, else 2 D).
inline int dense_row_bytes(int D, int dtype) { return (dtype == RB_I8 || dtype == RB_E4M3) ? D : 2 * D; }
int num_sms();
size_t dense_chunk_stride(const DensePlan& pl);
// mode 0: candidate pass over every tile; mode 1: sampling pass (one max per sampled tile).
int dense_scan_pass(int mode, int elem, const void* q, const void* x, int B, int N, int D, const DensePlan& pl,
                    int k, const float* seed, uint2* lists, int* counts, float* chunk_max, int* err,
                    cudaStream_t stream, const float* q_scale = nullptr, const float* x_scale = nullptr,
                    const FilterArgs* filter = nullptr, const int* qsg_live = nullptr);
// The same for two ranks at once (nseg 1, no values): out1 / out2 bound the k1-th / k2-th.
int row_kth2_lower_bounds(const float* vals, int B, int n, int64_t stride, int k1, int k2, float* out1, float* out2,
                          cudaStream_t stream);
// Per row of vals [B, n] (row stride `stride`): a lower bound on the k-th
// largest value (exact to 22 leading key bits), -inf when n < k.
int row_kth_lower_bound(const float* vals, int B, int n, int64_t stride, int nseg, int64_t seg_stride, int k,
                        float* out, float* out_vals, cudaStream_t stream);

// Merge of per-(query, split) candidate lists into the final sorted top-k.
// row_live (optional): only rows with a nonzero entry are written.
int merge_lists(const uint2* lists, const int* counts, int B, int n_lists, int stride, int k, int64_t id_offset,
                int64_t* out_ids, float* out_scores, uint2* out_pairs, cudaStream_t stream,
                const int* row_live = nullptr);
int merge_pair_stack(const uint2* pairs, int W, int B, int kin, int k, int64_t* out_ids, float* out_scores,
                     cudaStream_t stream);

void fill_empty(int64_t* out_ids, float* out_scores, size_t n, cudaStream_t stream);

// The int8 candidate scan (cand_scan.cu, kind 2): per query b, the exact top-k
// over the slots [0, counts[b]) of pos[b, :P] (positions into the int8 item
// table; a negative position is never scored), ranked on the raw score
// fp32(dot) (divisor -1) or fp16(dot / divisor), ties to the lower slot.
// Writes the winners' slots and raw scores, -1 / -inf past the candidates.
size_t cand_i8_ws_bytes(int B, int P, int k);
int cand_i8_max_k();
// With out_pairs not null the winners go there instead, as (raw score bits, slot) pairs.
int cand_i8_topk(const int8_t* q_codes, const int8_t* items, int N, int D, const int64_t* pos, int P,
                 const int64_t* counts, int B, int k, int divisor, int64_t* out_slots, float* out_raw, void* workspace,
                 cudaStream_t s, uint2* out_pairs = nullptr);

void fill_empty_pairs(uint2* out, size_t n, cudaStream_t stream);

// Bit-sliced Bloom words for the filtered dense scan (bloom.cu): bytes for N items
// (whole 128-item tiles) and the device build from the per-item words.
size_t bloom_slices_bytes(int64_t N);
int bloom_slices(const uint64_t* words, int64_t N, uint32_t* slices, cudaStream_t stream);

// Exact Hamming top-k by counting select (ham_select.cu), any k: over the N rows of
// `items` (pos null) or over each row's candidate slots pos[b, :counts[b]] (P wide).
// Ties go to the lower row / slot. W <= 16 words.
size_t ham_select_ws_bytes(int B, int L, int W, int k);
int ham_select_topk(const uint64_t* qbits, const uint64_t* items, int N, int W, const int64_t* pos, int P,
                    const int64_t* counts, int B, int k, int64_t* out_ids, float* out_scores, void* ws,
                    size_t ws_bytes, cudaStream_t s);

int merge_shard_lists(const int64_t* ids, const float* scores, int W, int B, int kin, int k, int64_t* out_ids,
                      float* out_scores, void* ws, cudaStream_t stream);
size_t merge_shard_ws_bytes(int W, int B, int kin);

// Caller-owned events recorded around the dominant kernel of the next call on
// this thread (profiling hook, see rb_set_profile_events).
struct ProfileEvents {
  cudaEvent_t start = nullptr, stop = nullptr;
};
ProfileEvents& profile_events();
// Records ev on the stream (inside a stream capture: as an external event node).
void record_profile_event(cudaEvent_t ev, cudaStream_t stream);

}  // namespace rb
