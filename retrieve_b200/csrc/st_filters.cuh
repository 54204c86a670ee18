// Per-position filter tests of st::search (the probe range of a cluster, SilverTorch's exact
// clause filter and its bloom on its own index and plans), host and device: the scan kernels
// of ivf_search.cu call them on the device; tests/native/st_filters_host.cu runs the same code
// on the CPU against the reference's fixtures.
#pragma once

#include <cstdint>

#ifdef __CUDACC__
#define RB_HD __host__ __device__
#else
#define RB_HD
#endif

namespace rb {

// The sorted positions [start, start + len) of cluster c with l items, clipped to [0, N); an
// invalid cluster id is an empty cluster.
RB_HD inline void probe_range_len(const int64_t* offsets, int64_t n_lists, int64_t N, int64_t c, int64_t l,
                                  int64_t& start, int64_t& len) {
  start = 0;
  len = 0;
  if (c < 0 || c >= n_lists) return;
  const int64_t s = offsets[c];
  if (s < 0 || s >= N || l <= 0) return;
  start = s;
  len = l < N - s ? l : N - s;
}

RB_HD inline void probe_range(const int64_t* offsets, const int64_t* sizes, int64_t n_lists, int64_t N, int64_t c,
                              int64_t& start, int64_t& len) {
  start = 0;
  len = 0;
  if (c < 0 || c >= n_lists) return;
  probe_range_len(offsets, n_lists, N, c, sizes[c], start, len);
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

RB_HD inline bool exact_pass(const ExactArgs& ex, const int32_t* __restrict__ q, int64_t doc) {
  for (int c = 0; c < ex.n_clauses; ++c) {
    const int32_t qv = q[c];
    if (qv == -1) continue;
    bool match = false;
    const int64_t s1 = ex.clause_slots[c + 1] < ex.rows ? ex.clause_slots[c + 1] : ex.rows;
    for (int64_t s = ex.clause_slots[c] > 0 ? ex.clause_slots[c] : 0; s < s1; ++s) {
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

// SilverTorch's bloom filter on its own index and prepared plans (the op's `plans`
// without the exact recheck; bloom_index_search_cuda.cu:304-349, 469-544). The index
// is bundle-major: docs in bundles of 2048 (32 columns of 64), bundle i holding
// B_i = bundle_b_offsets[i + 1] - bundle_b_offsets[i] bit rows; doc d's bit of row r is
// bit 63 - d % 64 of word (bundle_b_offsets[d / 2048] + r) * 32 + (d / 64) % 32. The
// plans blob holds, per plan slot, the parser's eight byte offsets (operators uint8,
// their parameter offsets int32, parameters int32, stored hashes uint64) into the data
// after the 8 * slots header words. A plan runs as a postfix stack over the doc's
// column word: a term ANDs the rows of its first k distinct positions hash % B_i among
// its hash_k hashes; AND / OR fold as many entries as their parameter range holds;
// NOT complements; EMPTY is all ones. Every offset and index is checked against the
// sizes passed in; a malformed plan fails the doc.
constexpr int kBloomMaxK = 10;    // MAX_K_V2
constexpr int kBloomStack = 16;   // deepest plan stack served
constexpr int kBundleColumns = 32;

struct BloomArgs {
  const uint64_t* index;  // null: no bloom filter
  int64_t index_words;
  const int64_t* bundle_offsets;  // [n_bundles + 1]
  int64_t n_bundles;
  const int64_t* blob;
  int64_t blob_words;
  int slots;
  const int64_t* plan_index;  // [B], or null: row b runs plan b
  int k, hash_k;
};

// Plan p evaluated on one 64-doc column of the index: bit 63 - i is doc 64 * column + i
// (high bit first). A malformed plan, a column past the index or an empty bundle gives 0.
RB_HD inline uint64_t bloom_plan_word(const BloomArgs& a, int64_t p, int64_t column) {
  if (p < 0 || p >= a.slots || column < 0) return 0;
  const int64_t data_bytes = (a.blob_words - 8 * static_cast<int64_t>(a.slots)) * 8;
  int64_t o[8];
  for (int i = 0; i < 8; ++i) o[i] = a.blob[8 * p + i];
  for (int i = 0; i < 8; i += 2)
    if (o[i] < 0 || o[i] > o[i + 1] || o[i + 1] > data_bytes) return 0;
  if ((o[2] & 3) || (o[6] & 7)) return 0;
  const uint8_t* data = reinterpret_cast<const uint8_t*>(a.blob + 8 * static_cast<int64_t>(a.slots));
  const uint8_t* ops = data + o[0];
  const int64_t n_ops = o[1] - o[0];
  const int32_t* op_off = reinterpret_cast<const int32_t*>(data + o[2]);
  const int64_t n_off = (o[3] - o[2]) / 4;
  const uint64_t* hashes = reinterpret_cast<const uint64_t*>(data + o[6]);
  const int64_t n_hash = (o[7] - o[6]) / 8;
  const int64_t bundle = column / kBundleColumns;
  if (bundle >= a.n_bundles) return 0;
  const int64_t b0 = a.bundle_offsets[bundle];
  const int64_t bb = a.bundle_offsets[bundle + 1] - b0;
  if (bb <= 0) return 0;
  const int64_t col = column % kBundleColumns;
  uint64_t stack[kBloomStack];
  int sp = 0;
  int64_t term = 0;
  for (int64_t j = 0; j < n_ops; ++j) {
    const uint8_t op = ops[j];
    if (op == 4) {  // TERM
      uint64_t w = ~0ull;
      if ((term + 1) * a.hash_k > n_hash) {
        w = 0;
      } else {
        const uint64_t* h = hashes + term * a.hash_k;
        int64_t used[kBloomMaxK];
        int resolved = 0;
        for (int q = 0; q < a.hash_k && resolved < a.k; ++q) {
          const int64_t pos = static_cast<int64_t>(h[q] % static_cast<uint64_t>(bb));
          bool dup = false;
          for (int i = 0; i < resolved; ++i) dup |= used[i] == pos;
          if (!dup) used[resolved++] = pos;
        }
        for (int i = 0; i < resolved; ++i) {
          const int64_t wi = (b0 + used[i]) * kBundleColumns + col;
          w &= (wi >= 0 && wi < a.index_words) ? a.index[wi] : 0ull;
        }
      }
      ++term;
      if (sp < kBloomStack) stack[sp++] = w; else return 0;
    } else if (op == 1 || op == 2) {  // AND, OR
      const int64_t children = j + 1 < n_off ? static_cast<int64_t>(op_off[j + 1]) - op_off[j] : 0;
      uint64_t acc = op == 1 ? ~0ull : 0ull;
      for (int64_t i = 0; i < children; ++i) {
        if (sp == 0) return 0;
        const uint64_t v = stack[--sp];
        acc = op == 1 ? (acc & v) : (acc | v);
      }
      if (sp < kBloomStack) stack[sp++] = acc; else return 0;
    } else if (op == 3) {  // NOT
      if (sp == 0) return 0;
      stack[sp - 1] = ~stack[sp - 1];
    } else if (op == 5) {  // EMPTY
      if (sp < kBloomStack) stack[sp++] = ~0ull; else return 0;
    }
  }
  return sp == 0 ? 0 : stack[sp - 1];
}

RB_HD inline bool bloom_pass(const BloomArgs& a, int64_t row, int64_t doc) {
  const int64_t p = a.plan_index ? a.plan_index[row] : row;
  return (bloom_plan_word(a, p, doc >> 6) >> (63 - (doc & 63))) & 1ull;
}

// fused_kmean_ann_with_partial_masks' filter (silvertorch/ops/csrc/fused_kmean_ann_cuda.cu
// :661-721, 800-845; the triple of bloom_index_search_batch_return_partial_response): probe j
// of row b keeps the i-th doc of its cluster range when bit first[b P + j] + i of the words
// from words[cumsum[b P + j - 1]] on (from words[0] for the first range) is set, bits counted
// high bit first (bloom_index_util.cuh:137-180). A bit past the words drops the doc.
// With rows (filtering_bit_index, fused_kmean_ann_cuda.cu:710-713) row b reads the ranges of
// mask row rows[b] < n_rows instead of its own (a row index outside drops every doc).
struct PartialMask {
  const int32_t* cumsum;  // [R P] inclusive column cumsum; null: no partial mask
  const int8_t* first;    // [R P] bit offset of each range's first doc
  const uint64_t* words;
  int64_t n_words;
  int P;
  const int64_t* rows = nullptr;  // [B] row -> mask row, or null: row b reads mask row b
  int64_t n_rows = 0;             // R, with rows
};

RB_HD inline bool partial_mask_pass(const PartialMask& m, int64_t b, int64_t j, int64_t i) {
  if (m.rows != nullptr) {
    b = m.rows[b];
    if (b < 0 || b >= m.n_rows) return false;
  }
  const int64_t idx = b * m.P + j;
  const int64_t base = idx == 0 ? 0 : m.cumsum[idx - 1];
  const int64_t bit = static_cast<int64_t>(m.first[idx]) + i;
  if (base < 0 || bit < 0) return false;
  const int64_t w = base + bit / 64;
  if (w >= m.n_words) return false;
  return (m.words[w] >> (63 - bit % 64)) & 1ull;
}

// The filters of one search: at most one of a full-N mask (high bit first), the exact
// clauses, the bloom plans.
struct FilterSet {
  const uint64_t* mask;
  int64_t mask_words;
  ExactArgs ex;
  BloomArgs bloom;
  // st::fused_kmean_ann's filtering_bit_index: row b reads mask row mask_rows[b] < mask_n_rows
  // (a row index outside drops every doc); null: mask row b
  const int64_t* mask_rows = nullptr;
  int64_t mask_n_rows = 0;
};

// BLOOM = false compiles the bloom test out (the scan kernels without a bloom filter keep
// their registers).
template <bool BLOOM>
RB_HD inline bool pos_passes(const FilterSet& f, int64_t row, int64_t position) {
  if (f.mask != nullptr) {
    int64_t mr = row;
    if (f.mask_rows != nullptr) {
      mr = f.mask_rows[row];
      if (mr < 0 || mr >= f.mask_n_rows) return false;
    }
    const int64_t w = position >> 6;
    if (w < f.mask_words && ((f.mask[mr * f.mask_words + w] >> (63 - (position & 63))) & 1ull) == 0) return false;
  }
  if (f.ex.attrs != nullptr && !exact_pass(f.ex, f.ex.query + row * f.ex.n_clauses, position)) return false;
  if constexpr (BLOOM) {
    if (f.bloom.index != nullptr && !bloom_pass(f.bloom, row, position)) return false;
  }
  return true;
}


// Clipped length of a probed cluster and its warp-aligned part: a cluster longer than the row
// contributes at most the row (width is a multiple of 32, so later slots land past it).
RB_HD inline void clipped_probe(const int64_t* offsets, const int64_t* sizes, int64_t n_lists, int64_t N, int64_t c,
                                int width, int64_t& start, int64_t& len, int64_t& full) {
  probe_range(offsets, sizes, n_lists, N, c, start, len);
  if (len > width) len = width;
  full = len / 32 * 32;
}

// One row's slot layout (the reference scorer's: every probed cluster's warp-aligned prefix in
// probe order, then every remainder in probe order; fused_kmean_ann_cuda.cu:100-110, 183-215):
// head[j] / tail[j] = the first head / tail slot of probe j; returns the row's slot total.
RB_HD inline int64_t row_slot_starts(const int64_t* prow, int P, const int64_t* offsets, const int64_t* sizes,
                                     int64_t n_lists, int64_t N, int width, int64_t* head, int64_t* tail) {
  int64_t h = 0;
  for (int j = 0; j < P; ++j) {
    int64_t start, len, full;
    clipped_probe(offsets, sizes, n_lists, N, prow[j], width, start, len, full);
    head[j] = h;
    h += full;
  }
  int64_t t = h;
  for (int j = 0; j < P; ++j) {
    int64_t start, len, full;
    clipped_probe(offsets, sizes, n_lists, N, prow[j], width, start, len, full);
    tail[j] = t;
    t += len - full;
  }
  return t;
}

// The probe of a slot (0 <= slot < row_total): the first j whose head (or tail) range ends past
// the slot, ends being the next probe's start (or the head total = tail[0], or row_total).
RB_HD inline int slot_to_probe(const int64_t* head, const int64_t* tail, int64_t row_total, int P, int64_t slot,
                               bool& in_head) {
  const int64_t total_head = tail[0];
  in_head = slot < total_head;
  int lo = 0, hi = P - 1;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    const int64_t end = in_head ? (mid + 1 < P ? head[mid + 1] : total_head) : (mid + 1 < P ? tail[mid + 1] : row_total);
    if (end > slot) hi = mid; else lo = mid + 1;
  }
  return lo;
}

}  // namespace rb
