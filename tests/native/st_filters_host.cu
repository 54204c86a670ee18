// Host entry points over the per-position filter tests of st::search
// (retrieve_b200/csrc/st_filters.cuh), so that the code the scan kernels run on the
// device can be checked on the CPU against the reference's fixtures
// (tests/test_st_filters_native.py builds this file with nvcc and loads it with ctypes).
#include <cstdint>

#include "st_filters.cuh"

using namespace rb;

extern "C" {

// out[i] = SilverTorch's bloom test of doc docs[i] for query row rows[i].
int host_bloom_pass(const int64_t* index, int64_t index_words, const int64_t* bundle_offsets, int64_t n_bundles,
                    const int64_t* blob, int64_t blob_words, int slots, const int64_t* plan_index, int k, int hash_k,
                    const int64_t* rows, const int64_t* docs, int64_t n, uint8_t* out) {
  const BloomArgs a{reinterpret_cast<const uint64_t*>(index), index_words, bundle_offsets, n_bundles, blob,
                    blob_words, slots, plan_index, k, hash_k};
  for (int64_t i = 0; i < n; ++i) out[i] = bloom_pass(a, rows[i], docs[i]) ? 1 : 0;
  return 0;
}

// out[q * n_cols + c] = plan q over column c (bloom_plan_word, the body of the device full
// search and partial search), for q < plan_count, c < n_cols.
int host_bloom_words(const int64_t* index, int64_t index_words, const int64_t* bundle_offsets, int64_t n_bundles,
                     const int64_t* blob, int64_t blob_words, int slots, int k, int hash_k, int plan_count,
                     int64_t n_cols, int64_t* out) {
  const BloomArgs a{reinterpret_cast<const uint64_t*>(index), index_words, bundle_offsets, n_bundles, blob,
                    blob_words, slots, nullptr, k, hash_k};
  for (int64_t q = 0; q < plan_count; ++q)
    for (int64_t c = 0; c < n_cols; ++c) out[q * n_cols + c] = static_cast<int64_t>(bloom_plan_word(a, q, c));
  return 0;
}

// out[i] = fused_kmean_ann_with_partial_masks' test of doc docs[i] of range (rows[i], probes[i]).
int host_partial_keep(const int32_t* cumsum, const int8_t* first, const int64_t* words, int64_t n_words, int P,
                      const int64_t* rows, const int64_t* probes, const int64_t* docs, int64_t n, uint8_t* out) {
  const PartialMask m{cumsum, first, reinterpret_cast<const uint64_t*>(words), n_words, P};
  for (int64_t i = 0; i < n; ++i) out[i] = partial_mask_pass(m, rows[i], probes[i], docs[i]) ? 1 : 0;
  return 0;
}

// out[i] = the exact clause test of doc docs[i] for query row rows[i].
int host_exact_pass(const int32_t* attrs, int64_t attr_rows, int64_t attr_docs, const int64_t* clause_slots,
                    const uint8_t* reverse, const int32_t* query, int n_clauses, const int64_t* rows,
                    const int64_t* docs, int64_t n, uint8_t* out) {
  const ExactArgs ex{attrs, attr_rows, attr_docs, clause_slots, reverse, query, n_clauses};
  for (int64_t i = 0; i < n; ++i) out[i] = exact_pass(ex, query + rows[i] * n_clauses, docs[i]) ? 1 : 0;
  return 0;
}

// out[i] = the full-N mask test (high bit first) of doc docs[i] for row rows[i], through pos_passes.
int host_mask_pass(const int64_t* mask, int64_t mask_words, const int64_t* rows, const int64_t* docs, int64_t n,
                   uint8_t* out) {
  FilterSet f{reinterpret_cast<const uint64_t*>(mask), mask_words,
              ExactArgs{nullptr, 0, 0, nullptr, nullptr, nullptr, 0},
              BloomArgs{nullptr, 0, nullptr, 0, nullptr, 0, 0, nullptr, 0, 0}};
  for (int64_t i = 0; i < n; ++i) out[i] = pos_passes<false>(f, rows[i], docs[i]) ? 1 : 0;
  return 0;
}

}  // extern "C"

extern "C" {

// The grouped and finish paths' slot arithmetic for one row: every slot below min(total, width)
// mapped back to its sorted position (row_slot_starts, slot_to_probe, clipped_probe); returns
// the row's slot total. head / tail: scratch of P entries each.
int64_t host_slot_positions(const int64_t* prow, int P, const int64_t* offsets, const int64_t* sizes, int64_t n_lists,
                            int64_t N, int width, int64_t* head, int64_t* tail, int64_t* positions) {
  const int64_t total = row_slot_starts(prow, P, offsets, sizes, n_lists, N, width, head, tail);
  for (int64_t slot = 0; slot < total && slot < width; ++slot) {
    bool in_head;
    const int j = slot_to_probe(head, tail, total, P, slot, in_head);
    int64_t start, len, full;
    clipped_probe(offsets, sizes, n_lists, N, prow[j], width, start, len, full);
    positions[slot] = start + (in_head ? slot - head[j] : full + (slot - tail[j]));
  }
  return total;
}

}  // extern "C"

#include "bloom_hash.cuh"

extern "C" {

// SilverTorch's bundle-major bloom index built on the CPU with the device build's functions
// (bloom_hash.cuh): widths and offsets (n_bundles + 1 entries, caller-sized), then the words
// (index: offsets[n_bundles] * 32 words, zeroed by the caller when index is not null).
int host_bloom_build(const int32_t* feature_ids, const int64_t* feature_offsets, const int64_t* feature_values,
                     int64_t N, int C, int k, double b_multiplier, int64_t fixed_b, int64_t* offsets,
                     uint64_t* index) {
  const int64_t n_bundles = (N + 2047) / 2048;
  offsets[0] = 0;
  for (int64_t i = 0; i < n_bundles; ++i) {
    int64_t m = 0;
    for (int64_t d = i * 2048; d < N && d < (i + 1) * 2048; ++d) {
      const int64_t cnt = feature_offsets[(d + 1) * C] - feature_offsets[d * C];
      m = cnt > m ? cnt : m;
    }
    offsets[i + 1] = offsets[i] + bloom_bundle_width(m, k, b_multiplier, fixed_b);
  }
  if (index == nullptr) return 0;
  for (int64_t d = 0; d < N; ++d) {
    const int64_t bundle = d / 2048;
    const int64_t b0 = offsets[bundle], bb = offsets[bundle + 1] - b0;
    if (bb <= 0) continue;
    for (int c = 0; c < C; ++c) {
      for (int64_t v = feature_offsets[d * C + c]; v < feature_offsets[d * C + c + 1]; ++v) {
        int64_t used[kBloomMaxBuildK];
        const int n_used = bloom_build_positions(static_cast<uint64_t>(static_cast<int64_t>(feature_ids[c])),
                                                 static_cast<uint64_t>(feature_values[v]), bb, k, used);
        for (int i = 0; i < n_used; ++i) index[bloom_word(b0, used[i], d)] |= bloom_bit(d);
      }
    }
  }
  return 0;
}

}  // extern "C"
