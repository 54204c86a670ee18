// st::search's scorer on the tensor cores (kind::i8): the grouped IVF scan with
// each task (a probed cluster and up to 128 of the (row, probe) pairs probing it)
// run as one M = 128 x N = 128 x K = D int8 MMA per 128-row tile of the cluster.
//
//  * tc_gather_kernel: per task, the pairs' int8 query codes gathered into rows
//    [128 t, 128 t + 128) of a [tasks x 128, D] block (zero rows past the
//    task's pairs), and the task's (cluster, first pair, pairs) record.
//  * ivf_tc_scan_kernel: one persistent CTA per SM, the dense scan's pipeline
//    shape: warp 0 loads the task's query block once and the cluster's row
//    tiles (TMA, 128-byte swizzle) through a STAGES-deep ring; warp 1 issues the
//    MMAs into a double-buffered TMEM accumulator (s32); warps 2-5 read one
//    pair's 128 dots a tile (thread = pair; the pairs dealt round the four
//    warps), keep the rows of the cluster that
//    land inside the row's width, rank them on the raw score (the int32 dot, or
//    fp16(dot / divisor)) and append (raw, slot) to the pair's list in
//    ascending slot order, testing the full-N mask or the exact clauses only
//    for the rows over the list's threshold; a list that fills is compacted to
//    the k best (ties to the lower slot) and its threshold rises.
// The lists then go through the same merge and slot -> id epilogue as the SIMT
// grouped scorer (ivf_search.cu), so the results are the row path's, bit for bit.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "dense_scan_kernels.cuh"
#include "st_filters.cuh"

namespace rb {

namespace {

constexpr int kTcRows = 128;      // pairs a task (MMA M) and cluster rows a tile (MMA N)
constexpr int kTcEpiWarps = 4;
constexpr int kTcThreads = 64 + 32 * kTcEpiWarps;

struct TcTask {
  int64_t cluster;
  int64_t p0;  // first pair (index into the cluster-grouped pair array)
  int32_t m;   // pairs in the task
  int32_t pad;
};

struct alignas(64) TcParams {
  CUtensorMap tmap_q;  // [tasks x 128, D] gathered query codes
  CUtensorMap tmap_x;  // [N, D] cluster-sorted item codes, 128-row boxes
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
  int* err;
};

template <int KB, int STAGES>
struct TcLayout {
  static constexpr int kOpTile = kTcRows * 128;
  static constexpr int kA = KB * kOpTile;
  static constexpr int kB = STAGES * KB * kOpTile;
  static constexpr int kHist = kTcEpiWarps * 256 * 4;
  static constexpr int kBar = (2 * STAGES + 2 + 4 + 1) * 8;
  static constexpr int kTotal = kA + kB + kHist + kBar + 16 + 1024;
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
  // pair r of the task goes to MMA row (r % 4) * 32 + r / 4: the task's pairs spread over the
  // four TMEM lane quadrants, so all four epilogue warps share their lists' work
  const int words = D / 16;  // D is a multiple of 128 here
  int4* dst = reinterpret_cast<int4*>(out + t * kTcRows * D);
  for (int i = threadIdx.x; i < kTcRows * words; i += blockDim.x) {
    const int row = i / words, w = i - row * words;
    const int r = (row & 31) * 4 + (row >> 5);
    int4 v = make_int4(0, 0, 0, 0);
    if (r < m) v = reinterpret_cast<const int4*>(q_codes + static_cast<int64_t>(pairs[p0 + r] / P) * D)[w];
    dst[i] = v;
  }
}

// Raw score of an int32 dot: the dot itself (divisor -1) or fp16(dot / divisor),
// the reference scorer's ranking value. Monotonic non-decreasing in the dot.
__device__ __forceinline__ float tc_raw(int dot, int divisor) {
  const float s = static_cast<float>(dot);  // exact: |dot| < 2^24 for D <= 512
  return divisor == -1 ? s : __half2float(__float2half_rn(__fdiv_rn(s, static_cast<float>(divisor))));
}

__device__ __forceinline__ int max32_s32(const uint32_t (&r)[32]) {
  int a[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = max(static_cast<int>(r[2 * i]), static_cast<int>(r[2 * i + 1]));
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
#pragma unroll
    for (int i = 0; i < w; ++i) a[i] = max(a[2 * i], a[2 * i + 1]);
  }
  return a[0];
}

template <int KB, int STAGES, int EPL, bool FILT>
__global__ void __launch_bounds__(kTcThreads, 1) ivf_tc_scan_kernel(const __grid_constant__ TcParams p) {
  using L = TcLayout<KB, STAGES>;
  constexpr int kKSteps = 4;  // 32-byte K steps per 128-byte K-block
  constexpr uint32_t kTmemCols = 2 * kTcRows;
  constexpr uint32_t kIdesc = make_idesc(2, 1, kTcRows, kTcRows);  // s32 accumulate, signed int8 operands

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + L::kA;
  uint32_t* hist_all = reinterpret_cast<uint32_t*>(smem + L::kA + L::kB);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kA + L::kB + L::kHist);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* a_full = bars + 2 * STAGES;
  uint64_t* a_empty = a_full + 1;
  uint64_t* acc_full = a_full + 2;   // [2]
  uint64_t* acc_empty = a_full + 4;  // [2]
  uint64_t* drain_bar = a_full + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t n_tasks = *p.n_tasks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
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
        if (a_iter > 0 && !mbar_wait(a_empty, (a_iter - 1) & 1, abort_flag)) {
          atomicCAS(p.err, 0, kDevTimeoutProducer);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(a_full, KB * L::kOpTile);
        for (int kb = 0; kb < KB; ++kb)
          tma_load_2d(smA + kb * L::kOpTile, &p.tmap_q, a_full, kb * 128, static_cast<int>(t * kTcRows));
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
      if (a_iter > 0) mbar_wait_drain(a_full, (a_iter - 1) & 1);
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
      const uint32_t a_base = smem_u32(smA), b_base = smem_u32(smB);
      for (int64_t t = blockIdx.x; t < n_tasks && !*abort_flag; t += gridDim.x) {
        int64_t start, len, full, p0;
        int m;
        task_range(t, start, len, full, m, p0);
        if (len == 0) continue;
        if (!mbar_wait(a_full, a_iter & 1, abort_flag)) {
          atomicCAS(p.err, 0, kDevTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        ++a_iter;
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
              const uint64_t ad = sw128_kmajor_desc(a_base + kb * L::kOpTile + j * 32);
              const uint64_t bd = sw128_kmajor_desc(b_base + (stage * KB + kb) * L::kOpTile + j * 32);
              mma_i8(d_col, ad, bd, kIdesc, (kb | j) != 0);
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
        mma_commit(a_empty);
      }
      mma_commit(drain_bar);
      mbar_wait_drain(drain_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    uint32_t* hist = hist_all + ew * 256;
    int acc = 0;
    uint32_t acc_phase = 0;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    for (int64_t t = blockIdx.x; t < n_tasks; t += gridDim.x) {
      int64_t start, len, full, p0;
      int m;
      task_range(t, start, len, full, m, p0);
      if (len == 0) continue;  // its pairs keep the zero count they start with
      const int r = lane * 4 + quad;  // the task's pair this lane scores (its MMA row: quad * 32 + lane)
      const bool valid = r < m;
      const int32_t pair = valid ? p.pairs[p0 + r] : 0;
      const int64_t b = pair / p.P;
      const int64_t hs = valid ? p.head[pair] : 0, ts = valid ? p.tail[pair] : 0;
      uint2* list = p.lists + static_cast<int64_t>(pair) * p.cap;
      int count = 0;
      float thresh = -INFINITY;
      const int tiles = static_cast<int>((len + kTcRows - 1) / kTcRows);
      bool ok = true;
      for (int tile = 0; tile < tiles; ++tile) {
        const bool need = valid && count > p.cap - kTcRows;  // room for a whole tile of appends
        if (__any_sync(RB_FULL_MASK, need)) warp_compact_lists<EPL>(list, count, thresh, need, p.k, hist);
        if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag)) {
          if (lane == 0) atomicCAS(p.err, 0, kDevTimeoutEpilogue);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        if (quad >= m) {  // no pair of this task in the warp's quadrant: release the tile at once
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[acc]);
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1;
          continue;
        }
        const uint32_t col0 = tmem_base + lane_addr + static_cast<uint32_t>(acc * kTcRows);
        uint32_t v[4][32];
        __syncwarp();
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) tmem_ld_32x32(col0 + ch * 32, v[ch]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
        // rows i0 .. i0 + 127 of the cluster; the row's slots of this tile all lie inside
        // the cluster and the width unless the tile is the cluster's last or the width cuts it
        const int64_t i0 = static_cast<int64_t>(tile) * kTcRows;
        const int64_t i_end = min(len, i0 + kTcRows);
        const int64_t last_slot = (i_end - 1) < full ? hs + (i_end - 1) : ts + (i_end - 1 - full);
        const bool clean = i_end - i0 == kTcRows && last_slot < p.width;
        int cm[4];
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) cm[ch] = max32_s32(v[ch]);
        bool any = false;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) any |= tc_raw(cm[ch], p.divisor) >= thresh;
        if (!__any_sync(RB_FULL_MASK, valid && any)) continue;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          if (!(valid && tc_raw(cm[ch], p.divisor) >= thresh)) continue;
          uint2* w = list + count;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int64_t i = i0 + ch * 32 + j;
            const float s = tc_raw(static_cast<int>(v[ch][j]), p.divisor);
            if (s >= thresh) {
              const int64_t slot = i < full ? hs + i : ts + (i - full);
              bool keep = clean || (i < len && slot < p.width);
              if constexpr (FILT) keep = keep && pos_passes<false>(p.f, b, start + i);
              if (keep) {
                *w = make_uint2(__float_as_uint(s), static_cast<uint32_t>(slot));
                ++w;
              }
            }
          }
          count = static_cast<int>(w - list);
        }
      }
      if (!ok) break;
      const bool need = valid && count > p.k;
      warp_compact_lists<EPL>(list, count, thresh, need, p.k, hist);
      if (valid) p.list_counts[pair] = count;
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

}  // namespace

bool ivf_tc_supported(int D, int k_sel, bool bloom) {
  return !bloom && (D == 128 || D == 256 || D == 512) && k_sel <= 1024;
}

// A pair's list holds k winners plus a whole tile of appends; the room past k + 128 spaces
// the compactions out (a list of 512 is compacted about once per 380 appends).
int ivf_tc_cap(int k_sel) { return k_sel <= 384 ? 512 : 1280; }

size_t ivf_tc_ws_bytes(int64_t n_pairs, int64_t n_lists, int D) {
  const int64_t tasks = (n_pairs + kTcRows - 1) / kTcRows + std::min(n_lists, n_pairs);
  return align_up(static_cast<size_t>(tasks) * kTcRows * D, 256) + align_up(static_cast<size_t>(tasks) * sizeof(TcTask), 256);
}

int ivf_tc_scan(const int8_t* q_codes, int B, int D, int P, const int8_t* item_codes, int64_t N,
                const int64_t* offsets, const int64_t* sizes, int64_t n_lists, const int32_t* pairs,
                const int64_t* cpo, const int64_t* ctask, const int64_t* head, const int64_t* tail, int width,
                int k_sel, int divisor, const FilterSet& fs, uint2* lists, int* list_counts, int* err, void* ws,
                cudaStream_t s) {
  const int64_t n_pairs = static_cast<int64_t>(B) * P;
  const int64_t max_tasks = (n_pairs + kTcRows - 1) / kTcRows + std::min(n_lists, n_pairs);
  if (max_tasks == 0) return RB_OK;
  uint8_t* w8 = static_cast<uint8_t*>(ws);
  int8_t* qblock = reinterpret_cast<int8_t*>(w8);
  TcTask* tasks = reinterpret_cast<TcTask*>(w8 + align_up(static_cast<size_t>(max_tasks) * kTcRows * D, 256));
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
  prm.err = err;
  const bool filt = fs.mask != nullptr || fs.ex.attrs != nullptr;
  const bool large = prm.cap > 256;
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
