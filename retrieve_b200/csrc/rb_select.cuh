// Exact top-k selection building blocks shared by every scan kernel.
//
// The scan kernels keep, per (query, split), an append-only candidate list in
// global memory: entries {score bits, item id} that passed the query's current
// threshold. When a list nears its capacity, the owning warp compacts it in
// place to its k best entries (radix select over the composite key) and raises
// the query's threshold. A split scans its items in ascending id order, so an
// item tied with the k-th entry on score always loses the tie: after an exact
// compaction the threshold becomes strict (next float above the k-th score).
//
// The merge kernel then selects, per query, the k best entries over all of its
// splits' lists (block-wide radix select), sorts them and writes the output.
#pragma once

#include "rb_common.cuh"

namespace rb {

// Warp-wide suffix-scan radix step over a 256-bin histogram in shared memory.
// Each lane owns bins [8*lane, 8*lane+8). Finds the digit d whose bucket holds
// the need-th largest element; returns d, the count strictly above it and the
// bucket's own count (all warp-uniform).
__device__ __forceinline__ void warp_find_digit(const uint32_t* hist, uint32_t need, uint32_t& digit,
                                                uint32_t& above_digit, uint32_t& in_digit) {
  const int lane = threadIdx.x & 31;
  uint32_t b[8];
  uint32_t total = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    b[j] = hist[8 * lane + j];
    total += b[j];
  }
  uint32_t incl = total;  // inclusive suffix sum over lanes >= lane
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    uint32_t v = __shfl_down_sync(RB_FULL_MASK, incl, off);
    if (lane + off < 32) incl += v;
  }
  const uint32_t above = incl - total;
  const bool here = (above < need) && (need <= incl);
  const uint32_t hb = __ballot_sync(RB_FULL_MASK, here);
  const int src = hb ? (__ffs(hb) - 1) : 0;
  uint32_t d = 0, a = 0, c = 0;
  if (lane == src) {
    uint32_t acc = above;
#pragma unroll
    for (int j = 7; j >= 0; --j) {
      if (acc + b[j] >= need) {
        d = 8 * lane + j;
        a = acc;
        c = b[j];
        break;
      }
      acc += b[j];
    }
  }
  digit = __shfl_sync(RB_FULL_MASK, d, src);
  above_digit = __shfl_sync(RB_FULL_MASK, a, src);
  in_digit = __shfl_sync(RB_FULL_MASK, c, src);
}

// Warp radix select over register-resident keys (EPL per lane, key 0 = empty
// slot, never selected because callers ask for need <= number of valid keys).
// Returns the cut: exactly `k` keys are >= cut.
template <int EPL>
__device__ __forceinline__ uint64_t warp_radix_cut(const uint64_t (&key)[EPL], const bool (&valid)[EPL], int k,
                                                   uint32_t* hist) {
  const int lane = threadIdx.x & 31;
  uint64_t prefix = 0, mask = 0;
  uint32_t need = static_cast<uint32_t>(k);
  for (int shift = 56; shift >= 0; shift -= 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) hist[8 * lane + j] = 0;
    __syncwarp();
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      if (valid[e] && (key[e] & mask) == prefix) atomicAdd(&hist[(key[e] >> shift) & 0xffu], 1u);
    }
    __syncwarp();
    uint32_t digit, above, in_digit;
    warp_find_digit(hist, need, digit, above, in_digit);
    __syncwarp();
    prefix |= static_cast<uint64_t>(digit) << shift;
    mask |= static_cast<uint64_t>(0xffu) << shift;
    need -= above;
    if (in_digit == need) break;  // every key with this prefix is in: cut is exact
  }
  return prefix;
}

__device__ __forceinline__ uint64_t warp_min_u64(uint64_t v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    uint64_t o = __shfl_xor_sync(RB_FULL_MASK, v, off);
    v = o < v ? o : v;
  }
  return v;
}

// Compacts, one lane at a time, the candidate list of every lane with `need`
// set: keeps its k best entries (in list order) and raises its threshold to
// just above the k-th score. `list`/`count`/`thresh` are the calling lane's own
// state. Requires count <= 32 * EPL and count > k for the lanes that need it.
// All 32 lanes must call it (warp-collective).
template <int EPL>
__device__ __noinline__ void warp_compact_lists(uint2* list, int& count, float& thresh, bool need, int k,
                                                uint32_t* hist) {
  const int lane = threadIdx.x & 31;
  uint32_t pending = __ballot_sync(RB_FULL_MASK, need);
  while (pending) {
    const int src = __ffs(pending) - 1;
    pending &= pending - 1;
    uint2* l = reinterpret_cast<uint2*>(
        __shfl_sync(RB_FULL_MASK, reinterpret_cast<unsigned long long>(list), src));
    const int cnt = __shfl_sync(RB_FULL_MASK, count, src);
    uint64_t key[EPL];
    bool valid[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int i = e * 32 + lane;
      valid[e] = i < cnt;
      key[e] = 0;
      if (valid[e]) {
        const uint2 v = l[i];
        key[e] = make_key(v.x, v.y);
      }
    }
    const uint64_t cut = warp_radix_cut<EPL>(key, valid, k, hist);
    // Stable in-place compaction: an entry moves to a slot <= its own.
    int out = 0;
    uint64_t kmin = ~0ull;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const bool keep = valid[e] && key[e] >= cut;
      const uint32_t b = __ballot_sync(RB_FULL_MASK, keep);
      if (keep) {
        l[out + __popc(b & lanemask_lt())] = key_to_entry(key[e]);
        kmin = key[e] < kmin ? key[e] : kmin;
      }
      out += __popc(b);
    }
    kmin = warp_min_u64(kmin);
    if (lane == src) {
      count = out;
      const uint32_t hi = static_cast<uint32_t>(kmin >> 32);
      // strict: a later item (higher id) tied with the k-th score loses the tie
      const float t = (hi == 0xffffffffu) ? ord2f(hi) : ord2f(hi + 1u);
      thresh = fmaxf(thresh, t);
    }
    __syncwarp();
  }
}

// Of the items id0 + j with bit j set in sel, those that pass query q's
// attribute predicate (bit j of the result). Touches no register array.
__device__ __forceinline__ uint32_t pred_pass_bits(const FilterArgs& f, int q, uint32_t id0, uint32_t sel,
                                                   const int64_t* tile_rows = nullptr, uint32_t tile0 = 0) {
  uint32_t out = 0;
  while (sel) {
    const int j = __ffs(sel) - 1;
    sel &= sel - 1;
    if (pred_pass(f, q, id0 + j, tile_rows, tile0)) out |= 1u << j;
  }
  return out;
}


// Of the items id0 + j with bit j set in sel, those that pass query q's exact
// (attribute) predicate; the Bloom form is not consulted. `tile_rows` / `tile0`: as
// pred_exact_item.
// `wterms` / `ent`, when not null: the calling lane's query's terms in the warp's shared
// table (kMaxTerms a lane) and their count; the rows then come from `tile_rows`.
__device__ __forceinline__ uint32_t pred_exact_bits(const FilterArgs& f, int q, uint32_t id0, uint32_t sel,
                                                    const int64_t* tile_rows = nullptr, uint32_t tile0 = 0,
                                                    const ExactTerm* wterms = nullptr, int ent = 0) {
  if (wterms != nullptr) {
    const ExactTerm* mine = wterms + (threadIdx.x & 31) * kMaxTerms;
    const int ca = f.C * f.A;
    uint32_t out = 0;
    while (sel) {
      const int j = __ffs(sel) - 1;
      sel &= sel - 1;
      if (pred_exact_row_sm(mine, ent, tile_rows + static_cast<size_t>(id0 + j - tile0) * ca, ca, f.A))
        out |= 1u << j;
    }
    return out;
  }
  const PredTerm* t = f.terms + static_cast<size_t>(q) * kMaxTerms;
  const int nt = f.n_terms[q];
  if (nt == 0) return sel;
  uint32_t out = 0;
  while (sel) {
    const int j = __ffs(sel) - 1;
    sel &= sel - 1;
    if (pred_exact_item(f, t, nt, id0 + j, tile_rows, tile0)) out |= 1u << j;
  }
  return out;
}

// Appends the entries s[j] >= thresh of a 32-item chunk (items id0 + j).
// Padding slots hold NaN, which never passes.
__device__ __forceinline__ void append_chunk_bits(uint2* list, int& count, float thresh, const uint32_t (&s)[32],
                                                  uint32_t id0) {
  uint2* w = list + count;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (__uint_as_float(s[j]) >= thresh) {
      *w = make_uint2(s[j], id0 + j);
      ++w;
    }
  }
  count = static_cast<int>(w - list);
}

// Appends, with the whole warp, the entries >= thresh of every (lane, chunk) whose bit ch is
// set in that lane's `pass`: r[ch][j] = the lane's score of item row0 + 32 ch + j, `list` =
// the lane's candidate list, `stage` = 32 words of the warp's shared scratch (16-byte
// aligned). The owning lane stages its chunk in shared memory; then lane j tests item j
// against the owner's threshold and the kept entries go to the owner's list in one
// coalesced store, in item order. Padding scores are NaN, which never passes. The code is
// one short loop per chunk position, instead of 32 predicated stores by one lane.
template <int NCH>
__device__ __forceinline__ void warp_append_chunks(uint2* list, int& count, float thresh,
                                                   const uint32_t (&r)[NCH][32], uint32_t pass, uint32_t row0,
                                                   uint32_t* stage) {
  const int lane = threadIdx.x & 31;
  uint4* stage4 = reinterpret_cast<uint4*>(stage);
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch) {
    uint32_t who = __ballot_sync(RB_FULL_MASK, (pass >> ch) & 1u);
    while (who != 0u) {
      const int src = __ffs(who) - 1;
      who &= who - 1u;
      if (lane == src) {
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4)
          stage4[j4] = make_uint4(r[ch][4 * j4], r[ch][4 * j4 + 1], r[ch][4 * j4 + 2], r[ch][4 * j4 + 3]);
      }
      __syncwarp();
      const uint32_t v = stage[lane];
      const bool keep = __uint_as_float(v) >= __shfl_sync(RB_FULL_MASK, thresh, src);
      const uint32_t kept = __ballot_sync(RB_FULL_MASK, keep);
      const int base = __shfl_sync(RB_FULL_MASK, count, src);
      uint2* dst = reinterpret_cast<uint2*>(
          __shfl_sync(RB_FULL_MASK, reinterpret_cast<unsigned long long>(list), src));
      if (keep) dst[base + __popc(kept & lanemask_lt())] = make_uint2(v, row0 + 32u * ch + lane);
      if (lane == src) count += __popc(kept);
      __syncwarp();  // every lane has read the staged chunk before the next one is written
    }
  }
}

// The filtered form of warp_append_chunks for one 32-item chunk (items id0 + j): `who` = the
// lanes whose chunk max reached their threshold, `bm` = each such lane's Bloom mask of the
// chunk from the bit-sliced words (all ones when the lane has none: `use_sl` false). For each
// such lane in turn the warp stages its scores, lane j keeps item j if it reaches the owner's
// threshold and passes the owner's predicate, and the kept entries go to the owner's list in
// one coalesced store (`tile_rows` / `tile0`: the tile's attribute rows in shared memory, as
// pred_exact_item; `wterms` / `ent`: as pred_exact_bits). The predicate work is spread over the items: lane j tests item j
// (the Bloom word or attributes of consecutive items, the owner's terms read by every lane at
// one address), instead of one lane walking the chunk's items one after another.
__device__ __forceinline__ void warp_filter_append(const FilterArgs& f, uint2* list, int& count, float thresh,
                                                   const uint32_t (&s)[32], uint32_t who, uint32_t bm, bool use_sl,
                                                   int q, uint32_t id0, uint32_t* stage,
                                                   const int64_t* tile_rows = nullptr, uint32_t tile0 = 0,
                                                   const ExactTerm* wterms = nullptr, int ent = 0) {
  const int lane = threadIdx.x & 31;
  uint4* stage4 = reinterpret_cast<uint4*>(stage);
  while (who != 0u) {
    const int src = __ffs(who) - 1;
    who &= who - 1u;
    if (lane == src) {
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) stage4[j4] = make_uint4(s[4 * j4], s[4 * j4 + 1], s[4 * j4 + 2], s[4 * j4 + 3]);
    }
    __syncwarp();
    const uint32_t v = stage[lane];
    const int qs = __shfl_sync(RB_FULL_MASK, q, src);
    const bool sliced = __shfl_sync(RB_FULL_MASK, static_cast<int>(use_sl), src) != 0;
    const uint32_t bms = __shfl_sync(RB_FULL_MASK, bm, src);
    const int ents = __shfl_sync(RB_FULL_MASK, ent, src);
    bool keep = __uint_as_float(v) >= __shfl_sync(RB_FULL_MASK, thresh, src) && ((bms >> lane) & 1u) != 0u;
    if (__any_sync(RB_FULL_MASK, keep) && keep) {
      const uint32_t id = id0 + static_cast<uint32_t>(lane);
      if (!sliced) {
        keep = pred_pass(f, qs, id, tile_rows, tile0);  // the item's Bloom word and / or attributes
      } else if (f.mode == kFilterBloomRecheck) {
        if (wterms != nullptr) {  // the owner's terms from the warp's table, the row from the ring
          const int ca = f.C * f.A;
          keep = pred_exact_row_sm(wterms + src * kMaxTerms, ents, tile_rows + static_cast<size_t>(id - tile0) * ca,
                                   ca, f.A);
        } else {
          keep = pred_exact_item(f, f.terms + static_cast<size_t>(qs) * kMaxTerms, f.n_terms[qs], id, tile_rows,
                                 tile0);
        }
      }
    }
    const uint32_t kept = __ballot_sync(RB_FULL_MASK, keep);
    const int base = __shfl_sync(RB_FULL_MASK, count, src);
    uint2* dst =
        reinterpret_cast<uint2*>(__shfl_sync(RB_FULL_MASK, reinterpret_cast<unsigned long long>(list), src));
    if (keep) dst[base + __popc(kept & lanemask_lt())] = make_uint2(v, id0 + static_cast<uint32_t>(lane));
    if (lane == src) count += __popc(kept);
    __syncwarp();  // every lane has read the staged chunk before the next one is written
  }
}

// Bit j set iff s[j] >= thresh. Every index into s is a compile-time constant,
// so the score array stays in registers.
__device__ __forceinline__ uint32_t chunk_pass_bits(const uint32_t (&s)[32], float thresh) {
  uint32_t m = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) m |= static_cast<uint32_t>(__uint_as_float(s[j]) >= thresh) << j;
  return m;
}

// Appends the entries of a 32-item chunk whose bit is set in mask.
__device__ __forceinline__ void append_chunk_mask(uint2* list, int& count, const uint32_t (&s)[32], uint32_t mask,
                                                  uint32_t id0) {
  uint2* w = list + count;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if ((mask >> j) & 1u) {
      *w = make_uint2(s[j], id0 + j);
      ++w;
    }
  }
  count = static_cast<int>(w - list);
}

// Three-input fp32 max (sm_100: one instruction). NaN operands are ignored
// as by fmaxf: the result is NaN only when all three are.
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Max of 32 fp32 values (raw bits): 16 instructions, three-input maxima in a
// tree of depth 4 (32 -> 11 -> 4 -> 2 -> 1). NaN entries are ignored.
__device__ __forceinline__ float max32(const uint32_t (&s)[32]) {
  float a[11];
#pragma unroll
  for (int i = 0; i < 10; ++i)
    a[i] = fmax3f(__uint_as_float(s[3 * i]), __uint_as_float(s[3 * i + 1]), __uint_as_float(s[3 * i + 2]));
  a[10] = fmaxf(__uint_as_float(s[30]), __uint_as_float(s[31]));
  const float b0 = fmax3f(a[0], a[1], a[2]), b1 = fmax3f(a[3], a[4], a[5]), b2 = fmax3f(a[6], a[7], a[8]);
  const float b3 = fmaxf(a[9], a[10]);
  return fmaxf(fmax3f(b0, b1, b2), b3);
}

// ---------------------------------------------------------------------------
// Threads of the block-level merge and select kernels.
// ---------------------------------------------------------------------------
constexpr int kMergeThreads = 256;

}  // namespace rb
