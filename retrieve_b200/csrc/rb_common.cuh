// Shared device helpers for the retrieve_b200 kernels: score keys with the
// "score descending, id ascending" total order, bounded mbarrier waits, and thin
// inline-PTX wrappers for the sm_100a async units (TMA, tcgen05 MMA / TMEM).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define RB_FULL_MASK 0xffffffffu

namespace rb {

// ---------------------------------------------------------------------------
// Error words written by kernels (device side) and returned by the C-ABI.
// ---------------------------------------------------------------------------
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutProducer = 1,   // TMA producer gave up waiting for a free stage
  kDevTimeoutMma = 2,        // MMA issuer gave up waiting for data / accumulator
  kDevTimeoutEpilogue = 3,   // epilogue gave up waiting for an accumulator
  kDevBadTmem = 4,           // TMEM allocation returned an unusable address
};

// A bounded wait gives up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// One lane of the (fully converged) warp returns true.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// Ordering keys.
// f2ord maps fp32 to uint32 so that a > b (IEEE compare, -0 == +0) iff
// f2ord(a) > f2ord(b). The composite 64-bit key puts the score in the high
// word and the complemented id in the low word: a larger key is a better item
// (higher score; on equal scores, lower id). Ids within one selection are
// distinct, so composite keys are distinct.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t f2ord_bits(uint32_t u) {
  if (u == 0x80000000u) u = 0u;  // -0 ranks with +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ uint32_t f2ord(float f) { return f2ord_bits(__float_as_uint(f)); }
__host__ __device__ __forceinline__ uint32_t ord2bits(uint32_t o) {
  return (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
}
__device__ __forceinline__ float ord2f(uint32_t o) { return __uint_as_float(ord2bits(o)); }

__device__ __forceinline__ uint64_t make_key(uint32_t score_bits, uint32_t id) {
  return (static_cast<uint64_t>(f2ord_bits(score_bits)) << 32) | static_cast<uint64_t>(~id);
}
__device__ __forceinline__ uint2 key_to_entry(uint64_t key) {
  return make_uint2(ord2bits(static_cast<uint32_t>(key >> 32)), ~static_cast<uint32_t>(key));
}

// ---------------------------------------------------------------------------
// Attribute predicates: per query up to kMaxTerms terms "clause c == value v",
// each possibly negated, combined as AND over groups of OR over the group's
// terms (conjunctive normal form; groups 0..7). A term matches an item exactly
// (some value of the item's clause c equals v; -1 pads) or through the item's
// 64-bit Bloom word (every bit of the term's mask set).
// ---------------------------------------------------------------------------
constexpr int kMaxTerms = 8;
struct PredTerm {        // 24 bytes, layout shared with the C-ABI rb_pred_term
  int64_t value;
  uint64_t bloom_mask;
  int32_t clause;
  int32_t flags;         // bits 0-2 group, bit 3 negate
};
enum FilterMode : int { kFilterNone = 0, kFilterExact = 1, kFilterBloom = 2, kFilterBloomRecheck = 3 };

struct FilterArgs {
  int mode;
  const PredTerm* terms;  // [B, kMaxTerms]
  const int* n_terms;     // [B]
  const int64_t* attrs;   // [N, C, A] int64, -1 pads (exact / recheck)
  int C, A;
  const uint64_t* bloom;  // [N] (bloom / recheck)
  // The same Bloom words bit-sliced, or null: per 32-item chunk 64 words, word p
  // holding bit p of the chunk's 32 items (bit j = item 32 chunk + j), whole
  // 128-item tiles (zero words past N). The scans then test a chunk's 32 items
  // against a term with one AND of the term's positions' words.
  const uint32_t* slices;
};

// A query's Bloom terms for the bit-sliced test, one word a term: bits 0-23 up
// to 4 bit positions (6 bits each), 24-26 their count, 27 negate, 28 last term
// of its group (the terms come grouped). `ok` is false when a term's mask has
// more than 4 bits or a group's terms are not contiguous: that query then uses
// the per-item test.
struct SlicedTerms {
  uint32_t t[kMaxTerms];
  int n;
  bool ok;
};

__device__ __forceinline__ SlicedTerms load_sliced_terms(const FilterArgs& f, int q, bool valid_q) {
  SlicedTerms st;
  st.n = valid_q ? min(f.n_terms[q], kMaxTerms) : 0;
  st.ok = true;
  const PredTerm* tm = f.terms + static_cast<size_t>(q) * kMaxTerms;
  uint32_t closed = 0;  // groups whose run of terms has ended
#pragma unroll
  for (int i = 0; i < kMaxTerms; ++i) {
    st.t[i] = 0;
    if (i < st.n) {
      uint64_t m = tm[i].bloom_mask;
      const int flags = tm[i].flags;
      const int bits = __popcll(m);
      if (bits > 4 || (closed >> (flags & 7)) & 1u) st.ok = false;  // wide mask, or a group split in two runs
      uint32_t w = 0;
      for (int j = 0; j < 4 && m != 0; ++j) {
        const int p = __ffsll(static_cast<long long>(m)) - 1;
        w |= static_cast<uint32_t>(p) << (6 * j);
        m &= m - 1;
      }
      w |= static_cast<uint32_t>(min(bits, 4)) << 24;
      if (flags & 8) w |= 1u << 27;
      const bool last = (i + 1 == st.n) || ((tm[i + 1].flags & 7) != (flags & 7));
      if (last) {
        w |= 1u << 28;
        closed |= 1u << (flags & 7);
      }
      st.t[i] = w;
    }
  }
  return st;
}

// Bit j set iff item j of the chunk passes the Bloom form of the predicate,
// from the chunk's 64 slice words `sl` (shared memory). An empty predicate
// passes everything.
__device__ __forceinline__ uint32_t bloom_chunk_mask(const uint32_t* sl, const SlicedTerms& st) {
  uint32_t res = 0xffffffffu, cur = 0;
#pragma unroll
  for (int i = 0; i < kMaxTerms; ++i) {
    if (i < st.n) {
      const uint32_t w = st.t[i];
      const int cnt = (w >> 24) & 7;
      // the four position words are read whatever the term's bit count (position 0 pads
      // the unused ones), so that the loads go out together
      const uint32_t a = sl[w & 63], b = sl[(w >> 6) & 63], c = sl[(w >> 12) & 63], d = sl[(w >> 18) & 63];
      uint32_t m = cnt > 0 ? a : 0xffffffffu;
      if (cnt > 1) m &= b;
      if (cnt > 2) m &= c;
      if (cnt > 3) m &= d;
      if (w & (1u << 27)) m = ~m;
      cur |= m;
      if (w & (1u << 28)) {
        res &= cur;
        cur = 0;
      }
    }
  }
  return res;
}

__device__ __forceinline__ bool pred_eval_one(const PredTerm* t, int nt, bool use_bloom, const int64_t* row,
                                              int A, uint64_t word) {
  uint32_t need = 0, got = 0;
  for (int i = 0; i < nt; ++i) {
    const PredTerm tm = t[i];
    const uint32_t g = 1u << (tm.flags & 7);
    need |= g;
    bool m;
    if (use_bloom) {
      m = (word & tm.bloom_mask) == tm.bloom_mask;
    } else {
      m = false;
      const int64_t* cell = row + static_cast<int64_t>(tm.clause) * A;
      for (int a = 0; a < A; ++a) m |= (cell[a] == tm.value);
    }
    if (tm.flags & 8) m = !m;
    if (m) got |= g;
  }
  return (got & need) == need;
}

// The exact form of pred_eval_one on one attribute row of ca <= 8 cells (global or shared
// memory), read whole before the first compare: the cells' loads are independent, so a
// recheck costs one memory round trip for the row instead of one per term (the query's
// terms stay in L1). The result is pred_eval_one's.
__device__ __forceinline__ bool pred_exact_row(const PredTerm* t, int nt, const int64_t* row, int ca, int A) {
  if (nt == 0) return true;
  int64_t cell[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) cell[c] = c < ca ? row[c] : 0;
  uint32_t need = 0, got = 0;
#pragma unroll 1
  for (int i = 0; i < nt; ++i) {
    const PredTerm tm = t[i];
    const uint32_t g = 1u << (tm.flags & 7);
    need |= g;
    bool m = false;
    const int lo = tm.clause * A;  // the clause's cells: lo .. lo + A - 1
#pragma unroll
    for (int c = 0; c < 8; ++c) m |= c < ca && c >= lo && c < lo + A && cell[c] == tm.value;
    if (tm.flags & 8) m = !m;
    if (m) got |= g;
  }
  return (got & need) == need;
}

// A term's exact test as the filtered 2-SM scan keeps it in shared memory, one table of
// kMaxTerms a query: lo = the clause's first cell (clause * A).
struct ExactTerm {
  int64_t value;
  int32_t lo;
  int32_t flags;
};

// pred_exact_row with the terms from such a table.
__device__ __forceinline__ bool pred_exact_row_sm(const ExactTerm* t, int nt, const int64_t* row, int ca, int A) {
  if (nt == 0) return true;
  int64_t cell[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) cell[c] = c < ca ? row[c] : 0;
  uint32_t need = 0, got = 0;
#pragma unroll 1
  for (int i = 0; i < nt; ++i) {
    const ExactTerm tm = t[i];
    const uint32_t g = 1u << (tm.flags & 7);
    need |= g;
    bool m = false;
#pragma unroll
    for (int c = 0; c < 8; ++c) m |= c < ca && c >= tm.lo && c < tm.lo + A && cell[c] == tm.value;
    if (tm.flags & 8) m = !m;
    if (m) got |= g;
  }
  return (got & need) == need;
}

// The exact predicate of terms t[0..nt) on item `id`: its row read whole when it has at
// most 8 cells, term by term (pred_eval_one) otherwise. `tile_rows`, when not null, holds
// the rows of the items tile0 .. tile0 + 127 in shared memory (the filtered scan's ring),
// which then serve instead of global memory.
__device__ __forceinline__ bool pred_exact_item(const FilterArgs& f, const PredTerm* t, int nt, uint32_t id,
                                                const int64_t* tile_rows = nullptr, uint32_t tile0 = 0) {
  if (nt == 0) return true;
  const int ca = f.C * f.A;
  if (ca > 8) return pred_eval_one(t, nt, false, f.attrs + static_cast<size_t>(id) * ca, f.A, 0ull);
  const int64_t* row = tile_rows != nullptr ? tile_rows + static_cast<size_t>(id - tile0) * ca
                                            : f.attrs + static_cast<size_t>(id) * ca;
  return pred_exact_row(t, nt, row, ca, f.A);
}

// Does item `id` pass query q's predicate?
// (`tile_rows` / `tile0`: as pred_exact_item.)
__device__ __forceinline__ bool pred_pass(const FilterArgs& f, int q, uint32_t id, const int64_t* tile_rows = nullptr,
                                          uint32_t tile0 = 0) {
  const PredTerm* t = f.terms + static_cast<size_t>(q) * kMaxTerms;
  const int nt = f.n_terms[q];
  if (nt == 0) return true;
  bool ok = true;
  if (f.mode == kFilterBloom || f.mode == kFilterBloomRecheck)
    ok = pred_eval_one(t, nt, true, nullptr, 0, f.bloom[id]);
  if (ok && (f.mode == kFilterExact || f.mode == kFilterBloomRecheck))
    ok = pred_exact_item(f, t, nt, id, tile_rows, tile0);
  return ok;
}

// ---------------------------------------------------------------------------
// cp.async (16-byte global -> shared copies, completed per thread).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Every committed group but the most recent one has landed.
__device__ __forceinline__ void cp_async_wait_group1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// ---------------------------------------------------------------------------
// mbarrier (shared::cta) with bounded waits.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return done != 0;
}
// Waits for the phase with the given parity to complete. Returns false when
// the wait ran past `limit_ns` (kWaitLimitNs unless a caller passes a shorter
// limit) or another role of the CTA raised `abort`.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint64_t limit_ns = kWaitLimitNs) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    // several tries between the abort / time checks keep a spinning warp's
    // issue slots for the warps that share its scheduler
#pragma unroll 1
    for (int i = 0; i < 16; ++i)
      if (mbar_try_wait(addr, parity)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// Bounded wait used on the exit path: ignores `abort` so that copies and MMAs
// already in flight land before the CTA releases its shared memory and TMEM.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), no multicast.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Untiled bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from
// global memory into this CTA's shared memory, completing on `bar`'s transaction count.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// Clusters (a CTA pair for the 2-SM MMA).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load of a CTA pair: lands in this CTA's shared memory and completes on
// the barrier at the same offset in CTA 0 of the pair (bit 24 of the
// shared::cluster address selects the peer).
constexpr uint32_t kPeerBitMask = 0xFEFFFFFFu;
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(smem_u32(bar) & kPeerBitMask), "r"(x), "r"(y)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads, fences.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// 2-SM MMA issued by CTA 0 of the pair: A rows / B rows split between the two
// CTAs' shared memory at the same offsets, D rows split between their TMEM.
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same for fp8 inputs (kind::f8f6f4; the formats come from the instruction
// descriptor: E4M3 for both operands here), fp32 accumulator.
__device__ __forceinline__ void mma_f8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives on the barrier at shared::cluster address `cluster_addr` (this CTA's
// or the peer's) once every prior tcgen05 op of this thread has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, f16/bf16 inputs.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same for signed 8-bit inputs with an s32 accumulator.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same for fp8 inputs (kind::f8f6f4, E4M3 operands by the descriptor).
__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives on `bar` once every tcgen05 op this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 columns of 32-bit: thread t of the warp receives row (lane base + t),
// columns [col, col + 16).
__device__ __forceinline__ void tmem_ld_32x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 32 columns of 32-bit: thread t of the warp receives row (lane base + t),
// columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA with
// 128-byte swizzle: rows of 128 bytes, 8-row swizzle atoms 1024 bytes apart.
// Bits: start>>4 [0,14), LBO>>4 [16,30) (unused by swizzled K-major, set to 1),
// SBO>>4 [32,46), version 1 [46,48), layout SWIZZLE_128B = 2 [61,64).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3ffffu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor: dense, K-major A and B, M x N tile.
//   c_format [4,6): 1 = f32, 2 = s32; a_format [7,10), b_format [10,13):
//   kind::f16 -> 0 = f16, 1 = bf16; kind::i8 -> 1 = signed.
//   n_dim [17,23) = N >> 3; m_dim [24,29) = M >> 4.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t c_format, uint32_t ab_format, uint32_t m, uint32_t n) {
  return (c_format << 4) | (ab_format << 7) | (ab_format << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

}  // namespace rb
