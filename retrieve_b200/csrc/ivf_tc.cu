// st::search's scorer on the tensor cores (kind::i8): the grouped IVF scan with
// each task (a probed cluster and up to 128 of the (row, probe) pairs probing it)
// run as one M = 128 cluster rows x N = (pairs, rounded up to 16) x K = D int8
// MMA per 128-row tile of the cluster.
//
//  * tc_gather_kernel: per task, the pairs' int8 query codes gathered into rows
//    [128 t, 128 t + m) of a [tasks x 128, D] block (zero rows after them), and
//    the task's (cluster, first pair, pairs) record.
//  * ivf_tc_scan_kernel: one persistent CTA per SM, the dense scan's pipeline
//    shape: warp 0 loads the task's query block once and the cluster's row
//    tiles (TMA, 128-byte swizzle) through a STAGES-deep ring; warp 1 issues the
//    MMAs (A = the cluster's rows, B = the pairs' queries) into a
//    double-buffered TMEM accumulator (s32: TMEM lane = cluster row, column =
//    pair); warps 2-5 each read 32 rows of the tile for every pair (thread =
//    row, 32 pairs a load) and, pair by pair, ballot the rows that land inside
//    the pair's row width and reach the pair's list threshold (compared on the
//    int32 dot: the smallest dot whose raw score reaches it), testing the
//    full-N mask or the exact clauses only for those rows; the passing rows are
//    appended to the pair's list together, at an offset taken from the pair's
//    shared count.
//  * Between tiles (named barrier of the 4 epilogue warps) each thread owns one
//    pair (pair j: warp j % 4, lane j / 4, so a task's compactions spread over
//    the warps): a list with less than a tile's room left is compacted to the k best
//    (ties to the lower slot: every later row of the pair has a higher slot, so
//    the threshold can be strict), and the row's bound is raised and read back:
//    a compacted list holds k candidates of its row at or above its k-th raw
//    score, so that score bounds the row's k-th from below and every pair of the
//    row may skip what falls under it (ties kept: another pair's rows may have
//    lower slots). Pairs of one row meet in different tasks, so the bound cuts
//    the appends the pairs of later tasks make.
// The lists then go through the same merge and slot -> id epilogue as the SIMT
// grouped scorer (ivf_search.cu), so the results are the row path's, bit for bit.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <climits>
#include <cstdint>
#include <cstring>

#include "dense_scan_kernels.cuh"
#include "st_filters.cuh"

namespace rb {

namespace {

constexpr int kTcRows = 128;   // cluster rows a tile (MMA M, TMEM lanes) and most pairs a task (MMA N)
constexpr int kTcEpiWarps = 4;
constexpr int kTcEpiThreads = 32 * kTcEpiWarps;
constexpr int kTcThreads = 64 + kTcEpiThreads;

struct TcTask {
  int64_t cluster;
  int64_t p0;  // first pair (index into the cluster-grouped pair array)
  int32_t m;   // pairs in the task
  int32_t pad;
};

// A pair's state during its task (shared memory). The first four words are read
// together for every (row, pair) test.
struct alignas(16) TcPair {
  int ithr;         // smallest int32 dot whose raw score reaches `thresh`
  uint32_t hlim;    // a head row i (i < full) lies inside the row's width iff i < hlim
  uint32_t tlim;    // a tail row i (i >= full) does iff i < tlim
  int count;        // entries in the pair's list
  float thresh;     // the list's threshold on the raw score (>=)
  uint32_t head32;  // slot of head row i: head32 + i (mod 2^32)
  uint32_t tail32;  // slot of tail row i: tail32 + i (mod 2^32)
  int pair;         // b * P + j
  int row;          // b
  int pad[3];
};

struct alignas(64) TcParams {
  CUtensorMap tmap_q;  // [tasks x 128, D] gathered query codes (B operand)
  CUtensorMap tmap_x;  // [N, D] cluster-sorted item codes (A operand), 128-row boxes
  const TcTask* tasks;
  const int64_t* n_tasks;  // device count (ctask[n_lists])
  const int32_t* pairs;    // pair ids b * P + j, grouped by cluster
  const int64_t* head;     // [B * P] first head slot of the pair's probe
  const int64_t* tail;     // [B * P] first tail slot
  const int64_t* offsets;
  const int64_t* sizes;
  int64_t n_lists, N;
  int P, width, k, cap, divisor;
  FilterSet f;  // full-N mask / exact clauses (no bloom plans on this path)
  uint2* lists;
  int* list_counts;
  uint32_t* row_bound;  // [B] f2ord of a lower bound on the row's k-th raw score (0: none yet)
  int* err;
};

// ABUF query blocks (two: the next task's block loads while the current one runs;
// one at D = 512, where two do not fit beside the row ring).
template <int KB, int STAGES>
struct TcLayout {
  static constexpr int kOpTile = kTcRows * 128;
  static constexpr int kABuf = KB == 4 ? 1 : 2;
  static constexpr int kA = KB * kOpTile;            // one query block
  static constexpr int kB = STAGES * KB * kOpTile;   // cluster row tiles
  static constexpr int kHist = kTcEpiWarps * 256 * 4;
  static constexpr int kPairs = kTcRows * static_cast<int>(sizeof(TcPair));
  static constexpr int kBar = (2 * STAGES + 2 * kABuf + 4 + 1) * 8;
  static constexpr int kTotal = kABuf * kA + kB + kHist + kPairs + kBar + 16 + 1024;
};

__global__ void tc_gather_kernel(const int8_t* __restrict__ q_codes, int D, int P, const int32_t* __restrict__ pairs,
                                 const int64_t* __restrict__ cpo, const int64_t* __restrict__ ctask, int64_t n_lists,
                                 int8_t* __restrict__ out, TcTask* __restrict__ tasks) {
  const int64_t t = blockIdx.x;
  if (t >= ctask[n_lists]) return;  // the grid bounds the task count from above
  int64_t lo = 0, hi = n_lists;     // the cluster: the largest c with ctask[c] <= t
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (ctask[mid] <= t) lo = mid; else hi = mid;
  }
  const int64_t p0 = cpo[lo] + (t - ctask[lo]) * kTcRows;
  const int m = static_cast<int>(min(static_cast<int64_t>(kTcRows), cpo[lo + 1] - p0));
  if (threadIdx.x == 0) tasks[t] = TcTask{lo, p0, m, 0};
  const int words = D / 16;  // D is a multiple of 128 here
  int4* dst = reinterpret_cast<int4*>(out + t * kTcRows * D);
  for (int i = threadIdx.x; i < kTcRows * words; i += blockDim.x) {
    const int r = i / words, w = i - r * words;
    int4 v = make_int4(0, 0, 0, 0);
    if (r < m) v = reinterpret_cast<const int4*>(q_codes + static_cast<int64_t>(pairs[p0 + r] / P) * D)[w];
    dst[i] = v;
  }
}

// Raw score of an int32 dot: the dot itself (divisor -1) or fp16(dot / divisor),
// the reference scorer's ranking value. Non-decreasing in the dot (divisor > 0).
__device__ __forceinline__ float tc_raw(int dot, int divisor) {
  const float s = static_cast<float>(dot);  // exact: |dot| < 2^24 for D <= 512
  return divisor == -1 ? s : __half2float(__float2half_rn(__fdiv_rn(s, static_cast<float>(divisor))));
}

// The smallest int32 dot d with tc_raw(d) >= thresh (INT_MIN: every dot does; INT_MAX:
// none does). |dot| < 2^24 for 8-bit codes and D <= 512.
__device__ int dot_threshold(float thresh, int divisor) {
  constexpr int kLim = 1 << 24;
  if (!(thresh > -INFINITY)) return INT_MIN;
  if (divisor == -1) {
    if (thresh > static_cast<float>(kLim)) return INT_MAX;
    if (thresh < -static_cast<float>(kLim)) return INT_MIN;
    return static_cast<int>(ceilf(thresh));  // float(d) is exact, so d >= thresh iff d >= ceil(thresh)
  }
  if (tc_raw(-kLim, divisor) >= thresh) return INT_MIN;
  if (tc_raw(kLim, divisor) < thresh) return INT_MAX;
  int lo = -kLim, hi = kLim;  // tc_raw(lo) < thresh <= tc_raw(hi)
  while (hi - lo > 1) {
    const int mid = lo + (hi - lo) / 2;
    if (tc_raw(mid, divisor) >= thresh) hi = mid; else lo = mid;
  }
  return hi;
}

// Named barrier 1 over the four epilogue warps, and its AND-reduction form.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kTcEpiThreads) : "memory"); }
__device__ __forceinline__ bool epi_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, 1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(kTcEpiThreads)
      : "memory");
  return r != 0;
}

// Between tiles: each thread owns pair `et` of the task (et < m). Raises the pair's
// threshold to the row's bound `rb`, compacts the list to the k best when it holds
// more than `limit` entries, publishes the compacted list's k-th score as the row's
// bound, and stores the state back (`last`: writes the list's count out instead).
// Called by every lane of the epilogue warps.
template <int EPL>
__device__ __forceinline__ void tc_pair_update(const TcParams& p, TcPair* sp, int et, int m, uint32_t rb, int limit,
                                               uint32_t* hist, bool last) {
  const bool mine = et < m;
  TcPair* s = sp + (mine ? et : 0);
  float th = mine ? fmaxf(s->thresh, ord2f(rb)) : -INFINITY;  // ord2f(0) is NaN: ignored
  int cnt = mine ? s->count : 0;
  uint2* list = p.lists + static_cast<int64_t>(mine ? s->pair : 0) * p.cap;
  const bool need = mine && cnt > limit;
  if (__any_sync(RB_FULL_MASK, need)) warp_compact_lists<EPL>(list, cnt, th, need, p.k, hist);
  // the strict threshold sits one step above the k-th score: one step below it is
  // that score (or, for a threshold raised by the bound, less than the bound)
  if (need) atomicMax(p.row_bound + s->row, f2ord(th) - 1u);
  if (mine) {
    if (last) {
      p.list_counts[s->pair] = cnt;
    } else {
      if (th != s->thresh) {
        s->thresh = th;
        s->ithr = dot_threshold(th, p.divisor);
      }
      s->count = cnt;
    }
  }
}

template <int KB, int STAGES, int EPL, bool FILT>
__global__ void __launch_bounds__(kTcThreads, 1) ivf_tc_scan_kernel(const __grid_constant__ TcParams p) {
  using L = TcLayout<KB, STAGES>;
  constexpr int kKSteps = 4;  // 32-byte K steps per 128-byte K-block
  constexpr uint32_t kTmemCols = 2 * kTcRows;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kABuf = L::kABuf;
  uint8_t* smA = smem;  // [kABuf] query blocks
  uint8_t* smB = smem + kABuf * L::kA;
  uint32_t* hist_all = reinterpret_cast<uint32_t*>(smB + L::kB);
  TcPair* sp = reinterpret_cast<TcPair*>(smB + L::kB + L::kHist);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smB + L::kB + L::kHist + L::kPairs);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* a_full = bars + 2 * STAGES;  // [kABuf]
  uint64_t* a_empty = a_full + kABuf;    // [kABuf]
  uint64_t* acc_full = a_empty + kABuf;  // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t n_tasks = *p.n_tasks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < kABuf; ++b) {
      mbar_init(&a_full[b], 1);
      mbar_init(&a_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kTcEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmap_q);
    tma_prefetch_desc(&p.tmap_x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // a task's cluster rows: [start, start + len), `full` of them in the warp-aligned head
  auto task_range = [&](int64_t t, int64_t& start, int64_t& len, int64_t& full, int& m, int64_t& p0) {
    const TcTask tk = p.tasks[t];
    m = tk.m;
    p0 = tk.p0;
    clipped_probe(p.offsets, p.sizes, p.n_lists, p.N, tk.cluster, p.width, start, len, full);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int a_iter = 0;
      uint32_t armed = 0;
      for (int64_t t = blockIdx.x; t < n_tasks && !*abort_flag; t += gridDim.x) {
        int64_t start, len, full, p0;
        int m;
        task_range(t, start, len, full, m, p0);
        if (len == 0) continue;
        const int slot = a_iter % kABuf;
        const uint32_t use = static_cast<uint32_t>(a_iter / kABuf);  // earlier fills of this block
        if (use > 0 && !mbar_wait(&a_empty[slot], (use - 1) & 1, abort_flag)) {
          atomicCAS(p.err, 0, kDevTimeoutProducer);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&a_full[slot], KB * L::kOpTile);
        for (int kb = 0; kb < KB; ++kb)
          tma_load_2d(smA + slot * L::kA + kb * L::kOpTile, &p.tmap_q, &a_full[slot], kb * 128,
                      static_cast<int>(t * kTcRows));
        ++a_iter;
        const int tiles = static_cast<int>((len + kTcRows - 1) / kTcRows);
        for (int tile = 0; tile < tiles; ++tile) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag)) {
            atomicCAS(p.err, 0, kDevTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], KB * L::kOpTile);
          for (int kb = 0; kb < KB; ++kb)
            tma_load_2d(smB + (stage * KB + kb) * L::kOpTile, &p.tmap_x, &full_bar[stage], kb * 128,
                        static_cast<int>(start + static_cast<int64_t>(tile) * kTcRows));
          ++armed;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      for (int b = 0; b < kABuf; ++b) {
        const int n_b = (a_iter + kABuf - 1 - b) / kABuf;  // fills of block b
        if (n_b > 0) mbar_wait_drain(&a_full[b], (n_b - 1) & 1);
      }
      for (int s = 0; s < STAGES; ++s) {
        const uint32_t n_s = armed / STAGES + (static_cast<uint32_t>(s) < armed % STAGES ? 1u : 0u);
        if (n_s > 0) mbar_wait_drain(&full_bar[s], (n_s - 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      int a_iter = 0;
      const uint32_t q_base = smem_u32(smA), x_base = smem_u32(smB);
      for (int64_t t = blockIdx.x; t < n_tasks && !*abort_flag; t += gridDim.x) {
        int64_t start, len, full, p0;
        int m;
        task_range(t, start, len, full, m, p0);
        if (len == 0) continue;
        // M = 128 cluster rows, N = the task's pairs rounded up to 16 (zero query rows past m)
        const uint32_t idesc = make_idesc(2, 1, kTcRows, static_cast<uint32_t>((m + 15) & ~15));
        const int slot = a_iter % kABuf;
        if (!mbar_wait(&a_full[slot], static_cast<uint32_t>(a_iter / kABuf) & 1, abort_flag)) {
          atomicCAS(p.err, 0, kDevTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        ++a_iter;
        const uint32_t qa = q_base + static_cast<uint32_t>(slot * L::kA);
        const int tiles = static_cast<int>((len + kTcRows - 1) / kTcRows);
        bool ok = true;
        for (int tile = 0; tile < tiles; ++tile) {
          if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag) ||
              !mbar_wait(&full_bar[stage], phase, abort_flag)) {
            atomicCAS(p.err, 0, kDevTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_col = tmem_base + static_cast<uint32_t>(acc * kTcRows);
#pragma unroll
          for (int kb = 0; kb < KB; ++kb) {
#pragma unroll
            for (int j = 0; j < kKSteps; ++j) {
              const uint64_t ad = sw128_kmajor_desc(x_base + (stage * KB + kb) * L::kOpTile + j * 32);
              const uint64_t bd = sw128_kmajor_desc(qa + kb * L::kOpTile + j * 32);
              mma_i8(d_col, ad, bd, idesc, (kb | j) != 0);
            }
          }
          mma_commit(&empty_bar[stage]);
          mma_commit(&acc_full[acc]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1;
        }
        if (!ok) break;
        mma_commit(&a_empty[slot]);
      }
      mma_commit(drain_bar);
      mbar_wait_drain(drain_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int et = threadIdx.x - 64;  // 0 .. 127: the pair this thread sets up at a task's start
    // the pair this thread owns at the updates: pairs dealt round the four warps, so the
    // compactions of a task with few pairs spread over all of them
    const int own = lane * kTcEpiWarps + ew;
    const int quad = warp & 3;        // TMEM lane quadrant this warp may access: rows 32 quad ..
    uint32_t* hist = hist_all + ew * 256;
    int acc = 0;
    uint32_t acc_phase = 0;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    // Tiles between two updates: a list holds at most `room` entries after an update
    // (compacted to k above it), so the U tiles up to the next one (128 appends a pair
    // each at most) fit its capacity.
    const int U = max(1, min(4, (p.cap - 2 * p.k) / kTcRows - 1));  // room >= 2k + 128: compactions stay rare
    const int room = p.cap - U * kTcRows;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < n_tasks && ok; t += gridDim.x) {
      int64_t start, len, full, p0;
      int m;
      task_range(t, start, len, full, m, p0);
      if (len == 0) continue;  // its pairs keep the zero count they start with
      const int n16 = (m + 15) >> 4;  // 16-pair column groups (the MMA's N / 16)
      epi_sync();                     // every thread is done with the previous task's pairs
      if (et < n16 * 16) {
        TcPair s;
        if (et < m) {
          s.pair = p.pairs[p0 + et];
          s.row = s.pair / p.P;
          const int64_t hs = p.head[s.pair], ts = p.tail[s.pair];
          s.count = 0;
          s.thresh = fmaxf(-INFINITY, ord2f(__ldcg(p.row_bound + s.row)));
          s.ithr = dot_threshold(s.thresh, p.divisor);
          s.hlim = static_cast<uint32_t>(min(full, max(int64_t{0}, static_cast<int64_t>(p.width) - hs)));
          s.tlim =
              static_cast<uint32_t>(full + min(len - full, max(int64_t{0}, static_cast<int64_t>(p.width) - ts)));
          s.head32 = static_cast<uint32_t>(hs);
          s.tail32 = static_cast<uint32_t>(ts - full);
        } else {  // a padding column of the last group: no row passes
          s = TcPair{};
          s.ithr = INT_MAX;
          s.thresh = INFINITY;
        }
        sp[et] = s;
      }
      epi_sync();
      const int tiles = static_cast<int>((len + kTcRows - 1) / kTcRows);
      bool failed = false;  // this warp's wait ran out: it skips to the next update, where all stop
      for (int tile = 0; tile < tiles; ++tile) {
        const bool last = tile == tiles - 1;
        const bool update = last || tile % U == U - 1;
        // the row's bound for this thread's pair, read while the tile's MMA runs
        const uint32_t rb = (update && own < m) ? __ldcg(p.row_bound + sp[own].row) : 0u;
        if (!failed) failed = !mbar_wait(&acc_full[acc], acc_phase, abort_flag);
        if (!failed) {
          tc_fence_after();
          // this thread's cluster row (< 2^31 + 128: rows and limits stay in uint32)
          const uint32_t i = static_cast<uint32_t>(tile) * kTcRows + quad * 32 + lane;
          const bool in_head = static_cast<int64_t>(i) < full;
          const uint32_t col0 = tmem_base + lane_addr + static_cast<uint32_t>(acc * kTcRows);
#pragma unroll 1
          for (int g = 0; g < n16; ++g) {
            uint32_t v[16];
            __syncwarp();
            tmem_ld_32x16(col0 + g * 16, v);
            tmem_wait_ld();
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int j = g * 16 + jj;
              const int4 st = *reinterpret_cast<const int4*>(sp + j);  // ithr, hlim, tlim, count
              const int d = static_cast<int>(v[jj]);
              bool pass = i < (in_head ? static_cast<uint32_t>(st.y) : static_cast<uint32_t>(st.z)) && d >= st.x;
              if constexpr (FILT) {
                if (pass) pass = pos_passes<false>(p.f, sp[j].row, start + i);
              }
              const uint32_t bal = __ballot_sync(RB_FULL_MASK, pass);
              if (bal != 0u) {
                int base = 0;
                if (lane == 0) base = atomicAdd(&sp[j].count, __popc(bal));
                base = __shfl_sync(RB_FULL_MASK, base, 0);
                if (pass) {
                  const uint32_t slot = (in_head ? sp[j].head32 : sp[j].tail32) + i;
                  p.lists[static_cast<int64_t>(sp[j].pair) * p.cap + base + __popc(bal & lanemask_lt())] =
                      make_uint2(__float_as_uint(tc_raw(d, p.divisor)), slot);
                }
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
        if (update) {
          // every append of the tiles since the last update is in; the same decision in all
          // four warps, so no one is left at a barrier
          if (!epi_all(!failed)) {
            if (failed && lane == 0) atomicCAS(p.err, 0, kDevTimeoutEpilogue);
            *abort_flag = 1;
            ok = false;
            break;
          }
          // the row's bound, the thresholds, and room for the next U tiles (or, after the
          // last, the k best and the list's count)
          tc_pair_update<EPL>(p, sp, own, m, rb, last ? p.k : room, hist, last);
          if (!last) epi_sync();
        }
      }
    }
  }

  __syncwarp();
  if (*abort_flag) {
    // error path only: a load of this CTA may still be in flight; let it land
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) __nanosleep(10000);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int KB, int STAGES, int EPL, bool FILT>
cudaError_t launch_tc(const TcParams& prm, int grid, cudaStream_t s) {
  using L = TcLayout<KB, STAGES>;
  auto kern = ivf_tc_scan_kernel<KB, STAGES, EPL, FILT>;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  if (e != cudaSuccess) return e;
  kern<<<grid, kTcThreads, L::kTotal, s>>>(prm);
  return cudaGetLastError();
}

template <int KB, int STAGES>
cudaError_t launch_tc_kb(const TcParams& prm, bool filt, bool large, int grid, cudaStream_t s) {
  if (large) return filt ? launch_tc<KB, STAGES, 40, true>(prm, grid, s) : launch_tc<KB, STAGES, 40, false>(prm, grid, s);
  return filt ? launch_tc<KB, STAGES, 16, true>(prm, grid, s) : launch_tc<KB, STAGES, 16, false>(prm, grid, s);
}

size_t tc_query_block_bytes(int64_t max_tasks, int D) {
  return align_up(static_cast<size_t>(max_tasks) * kTcRows * D, 256);
}

}  // namespace

bool ivf_tc_supported(int D, int k_sel, bool bloom) {
  return !bloom && (D == 128 || D == 256 || D == 512) && k_sel <= 1024;
}

// A pair's list holds k winners plus the appends of the tiles between two updates (one tile
// at these sizes: the thresholds rise at every tile, which keeps the appends few).
int ivf_tc_cap(int k_sel) { return k_sel <= 384 ? 512 : 1280; }

// Gathered query blocks | task records.
size_t ivf_tc_ws_bytes(int64_t n_pairs, int64_t n_lists, int D) {
  const int64_t tasks = (n_pairs + kTcRows - 1) / kTcRows + std::min(n_lists, n_pairs);
  return tc_query_block_bytes(tasks, D) + align_up(static_cast<size_t>(tasks) * sizeof(TcTask), 256);
}

int ivf_tc_scan(const int8_t* q_codes, int B, int D, int P, const int8_t* item_codes, int64_t N,
                const int64_t* offsets, const int64_t* sizes, int64_t n_lists, const int32_t* pairs,
                const int64_t* cpo, const int64_t* ctask, const int64_t* head, const int64_t* tail, int width,
                int k_sel, int divisor, const FilterSet& fs, uint2* lists, int* list_counts, uint32_t* row_bound,
                int* err, void* ws, cudaStream_t s) {
  const int64_t n_pairs = static_cast<int64_t>(B) * P;
  const int64_t max_tasks = (n_pairs + kTcRows - 1) / kTcRows + std::min(n_lists, n_pairs);
  if (max_tasks == 0) return RB_OK;
  uint8_t* w8 = static_cast<uint8_t*>(ws);
  int8_t* qblock = reinterpret_cast<int8_t*>(w8);
  const size_t task_off = tc_query_block_bytes(max_tasks, D);
  TcTask* tasks = reinterpret_cast<TcTask*>(w8 + task_off);
  tc_gather_kernel<<<static_cast<unsigned>(max_tasks), 256, 0, s>>>(q_codes, D, P, pairs, cpo, ctask, n_lists, qblock,
                                                                      tasks);
  if (cudaGetLastError() != cudaSuccess) {
    set_last_error("st::search (tensor cores): gather launch failed");
    return RB_ERR_CUDA;
  }
  TcParams prm;
  std::memset(&prm, 0, sizeof(prm));
  if (!make_tmap_2d(&prm.tmap_q, qblock, 2, static_cast<uint64_t>(max_tasks) * kTcRows, static_cast<uint64_t>(D),
                    kTcRows) ||
      !make_tmap_2d(&prm.tmap_x, item_codes, 2, static_cast<uint64_t>(N), static_cast<uint64_t>(D), kTcRows)) {
    set_last_error("st::search (tensor cores): cuTensorMapEncodeTiled failed");
    return RB_ERR_CUDA;
  }
  prm.tasks = tasks;
  prm.n_tasks = ctask + n_lists;
  prm.pairs = pairs;
  prm.head = head;
  prm.tail = tail;
  prm.offsets = offsets;
  prm.sizes = sizes;
  prm.n_lists = n_lists;
  prm.N = N;
  prm.P = P;
  prm.width = width;
  prm.k = k_sel;
  prm.cap = ivf_tc_cap(k_sel);
  prm.divisor = divisor;
  prm.f = fs;
  prm.lists = lists;
  prm.list_counts = list_counts;
  prm.row_bound = row_bound;
  prm.err = err;
  const bool filt = fs.mask != nullptr || fs.ex.attrs != nullptr;
  const bool large = prm.cap > 512;  // lists of 1280: 40 entries a lane in the compaction (else 16)
  const int grid = static_cast<int>(std::min<int64_t>(max_tasks, num_sms()));
  cudaError_t e;
  if (D == 128)
    e = launch_tc_kb<1, 8>(prm, filt, large, grid, s);
  else if (D == 256)
    e = launch_tc_kb<2, 4>(prm, filt, large, grid, s);
  else
    e = launch_tc_kb<4, 2>(prm, filt, large, grid, s);
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

}  // namespace rb
