// Exact 1-bit Hamming top-k for k beyond the list kernels' limits (the full scan
// above k = 1024, the candidate scan above min(k, P) = 224): a counting select.
//
// A Hamming score 64 W - 2 h is decided by the distance h in [0, 64 W], so the
// exact order (score descending, index ascending) is: every item of distance 0
// in index order, then distance 1, and so on. Per query:
//   1. hist:      the count of items at every distance (shared-memory histograms
//                 of a block of items, added into [B, R]);
//   2. threshold: the distance T at which the running count reaches k; the
//                 items below T all win, `need` = k - (items below T) of the
//                 items at T win, the lowest indices first;
//   3. count:     per 4096-item block, its items below T and at T;
//   4. scan:      exclusive prefix of those counts over the blocks, in index
//                 order;
//   5. write:     each block writes its winners in index order at the offsets of
//                 step 4 (items below T after the ones of earlier blocks; items
//                 at T at `below + tie rank` while the tie rank is under `need`);
//   6. order:     one warp per query puts the k winners in distance order by a
//                 stable counting sort (index order kept within a distance), and
//                 writes ids, scores and the -1 / -inf pads.
// The full scan's items are the table's rows (index = row id); the candidate
// scan's are the row's candidate slots p < counts[b] (index = slot, id =
// positive_indices[b, p]; ids outside [0, N) are skipped), as the list kernels
// order them. Memory: [B, R] + [B, nblk, 4] ints and [B, k] pairs.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "rb_capi_internal.h"

namespace rb {

namespace {

constexpr int kHsBlock = 4096;   // items per block of steps 1, 3 and 5
constexpr int kHsThreads = 256;  // threads of those kernels (16 items each)

struct HamSel {
  const uint64_t* qbits;   // [B, W]
  const uint64_t* items;   // [N, W]
  const int64_t* pos;      // candidate scan: [B, P] ids; full scan: null
  const int64_t* counts;   // candidate scan: [B] (null: P each)
  int B, N, W, L;          // L: items a query ranks (N, or P)
  int k;                   // winners a query keeps (columns written)
  int R;                   // 64 W + 1 distances
  int nblk;                // ceil(L / kHsBlock)
  int* hist;               // [B, R]
  int* thr;                // [B, 4]: T, below, need, valid
  int* bcnt;               // [B, nblk, 2]: below, at
  int* boff;               // [B, nblk, 2]
  uint2* win;              // [B, k]: (distance, index)
};

// Distance of item `i` (a row, or a candidate slot) from query q; -1 when the
// slot holds no candidate.
__device__ __forceinline__ int ham_distance(const HamSel& a, const uint64_t* q, int qi, int i) {
  int64_t id = i;
  if (a.pos != nullptr) {
    const int64_t n_valid = a.counts != nullptr ? a.counts[qi] : a.L;
    if (i >= n_valid) return -1;
    id = a.pos[static_cast<int64_t>(qi) * a.L + i];
    if (id < 0 || id >= a.N) return -1;
  }
  const uint64_t* x = a.items + id * a.W;
  int h = 0;
  for (int w = 0; w < a.W; ++w) h += __popcll(q[w] ^ __ldg(x + w));
  return h;
}

// Step 1. grid (nblk, query groups of qg); shared: qg * R ints, then the group's query words.
__global__ void __launch_bounds__(kHsThreads) ham_hist_kernel(HamSel a, int qg) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  int* h_sm = reinterpret_cast<int*>(sm_raw);
  uint64_t* q_sm = reinterpret_cast<uint64_t*>(sm_raw + (static_cast<size_t>(qg) * a.R * 4 + 15) / 16 * 16);
  const int q0 = blockIdx.y * qg, nq = min(qg, a.B - q0);
  for (int i = threadIdx.x; i < nq * a.R; i += blockDim.x) h_sm[i] = 0;
  for (int i = threadIdx.x; i < nq * a.W; i += blockDim.x) q_sm[i] = a.qbits[static_cast<int64_t>(q0) * a.W + i];
  __syncthreads();
  const int lo = blockIdx.x * kHsBlock, hi = min(a.L, lo + kHsBlock);
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x)
    for (int j = 0; j < nq; ++j) {
      const int h = ham_distance(a, q_sm + j * a.W, q0 + j, i);
      if (h >= 0) atomicAdd(&h_sm[j * a.R + h], 1);
    }
  __syncthreads();
  for (int i = threadIdx.x; i < nq * a.R; i += blockDim.x)
    if (h_sm[i] != 0) atomicAdd(&a.hist[static_cast<int64_t>(q0) * a.R + i], h_sm[i]);
}

// Step 2. One thread per query.
__global__ void ham_threshold_kernel(HamSel a) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= a.B) return;
  const int* h = a.hist + static_cast<int64_t>(b) * a.R;
  int below = 0, t = a.R, need = 0;
  for (int d = 0; d < a.R; ++d) {
    if (below + h[d] >= a.k) {
      t = d;
      need = a.k - below;
      break;
    }
    below += h[d];
  }
  int* o = a.thr + 4 * b;
  o[0] = t;                        // distance of the last winners (R: every valid item wins)
  o[1] = below;                    // winners closer than t
  o[2] = need;                     // winners at t, lowest indices first
  o[3] = t < a.R ? a.k : below;    // winners in all (< k when fewer items are valid)
}

// Block-wide exclusive prefix of two 0/1 flags over the block's threads in
// thread order; returns the block totals.
__device__ __forceinline__ int2 block_rank2(bool f0, bool f1, int& r0, int& r1, int2* warp_sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t b0 = __ballot_sync(RB_FULL_MASK, f0), b1 = __ballot_sync(RB_FULL_MASK, f1);
  const uint32_t lt = lanemask_lt();
  if (lane == 0) warp_sm[warp] = make_int2(__popc(b0), __popc(b1));
  __syncthreads();
  int2 before = make_int2(0, 0), total = make_int2(0, 0);
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
    const int2 c = warp_sm[w];
    if (w < warp) {
      before.x += c.x;
      before.y += c.y;
    }
    total.x += c.x;
    total.y += c.y;
  }
  __syncthreads();  // warp_sm is reused by the next call
  r0 = before.x + __popc(b0 & lt);
  r1 = before.y + __popc(b1 & lt);
  return total;
}

// Steps 3 (WRITE = false) and 5 (WRITE = true). grid (nblk, query groups of qg).
template <bool WRITE>
__global__ void __launch_bounds__(kHsThreads) ham_block_kernel(HamSel a, int qg) {
  __shared__ int2 warp_sm[kHsThreads / 32];
  extern __shared__ __align__(16) unsigned char sm_raw[];
  uint64_t* q_sm = reinterpret_cast<uint64_t*>(sm_raw);
  const int q0 = blockIdx.y * qg, nq = min(qg, a.B - q0);
  for (int i = threadIdx.x; i < nq * a.W; i += blockDim.x) q_sm[i] = a.qbits[static_cast<int64_t>(q0) * a.W + i];
  __syncthreads();
  const int lo = blockIdx.x * kHsBlock, hi = min(a.L, lo + kHsBlock);
  for (int j = 0; j < nq; ++j) {
    const int b = q0 + j;
    const int* t = a.thr + 4 * b;
    const int T = t[0], below = t[1], need = t[2];
    int2 base = make_int2(0, 0);
    if (WRITE) {
      const int* o = a.boff + (static_cast<int64_t>(b) * a.nblk + blockIdx.x) * 2;
      base = make_int2(o[0], o[1]);
    }
    // items in index order, one per thread per round (all threads take part in every round)
    for (int r0 = lo; r0 < hi; r0 += blockDim.x) {
      const int i = r0 + threadIdx.x;
      const int h = i < hi ? ham_distance(a, q_sm + j * a.W, b, i) : -1;
      const bool is_below = h >= 0 && h < T, is_at = h >= 0 && h == T;
      int rb = 0, ra = 0;
      const int2 tot = block_rank2(is_below, is_at, rb, ra, warp_sm);
      if (WRITE) {
        uint2* w = a.win + static_cast<int64_t>(b) * a.k;
        if (is_below) w[base.x + rb] = make_uint2(static_cast<uint32_t>(h), static_cast<uint32_t>(i));
        if (is_at && base.y + ra < need)
          w[below + base.y + ra] = make_uint2(static_cast<uint32_t>(h), static_cast<uint32_t>(i));
      }
      base.x += tot.x;
      base.y += tot.y;
    }
    if (!WRITE && threadIdx.x == 0) {
      int* c = a.bcnt + (static_cast<int64_t>(b) * a.nblk + blockIdx.x) * 2;
      c[0] = base.x;
      c[1] = base.y;
    }
  }
}

// Step 4. One block per query: exclusive prefix over the blocks, both counters.
__global__ void __launch_bounds__(1024) ham_scan_kernel(HamSel a) {
  __shared__ int2 part[1024];
  const int b = blockIdx.x;
  const int n = a.nblk;
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int lo = min(n, threadIdx.x * per), hi = min(n, lo + per);
  const int* c = a.bcnt + static_cast<int64_t>(b) * n * 2;
  int2 s = make_int2(0, 0);
  for (int i = lo; i < hi; ++i) {
    s.x += c[2 * i];
    s.y += c[2 * i + 1];
  }
  part[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int2 run = make_int2(0, 0);
    for (int t = 0; t < static_cast<int>(blockDim.x); ++t) {
      const int2 v = part[t];
      part[t] = run;
      run.x += v.x;
      run.y += v.y;
    }
  }
  __syncthreads();
  int2 run = part[threadIdx.x];
  int* o = a.boff + static_cast<int64_t>(b) * n * 2;
  for (int i = lo; i < hi; ++i) {
    o[2 * i] = run.x;
    o[2 * i + 1] = run.y;
    run.x += c[2 * i];
    run.y += c[2 * i + 1];
  }
}

// Step 6. One warp per query: stable counting sort of its winners by distance.
__global__ void __launch_bounds__(32) ham_order_kernel(HamSel a, int64_t* out_ids, float* out_scores) {
  extern __shared__ int start[];  // [R]
  const int b = blockIdx.x, lane = threadIdx.x;
  const int* t = a.thr + 4 * b;
  const int n_win = t[3];
  const uint2* w = a.win + static_cast<int64_t>(b) * a.k;
  for (int d = lane; d < a.R; d += 32) start[d] = 0;
  __syncwarp();
  for (int i = lane; i < n_win; i += 32) atomicAdd(&start[w[i].x], 1);
  __syncwarp();
  if (lane == 0) {
    int run = 0;
    for (int d = 0; d < a.R; ++d) {
      const int c = start[d];
      start[d] = run;
      run += c;
    }
  }
  __syncwarp();
  int64_t* ids = out_ids + static_cast<int64_t>(b) * a.k;
  float* sc = out_scores + static_cast<int64_t>(b) * a.k;
  const int bits = 64 * a.W;
  const uint32_t lt = lanemask_lt();
  for (int c0 = 0; c0 < n_win; c0 += 32) {
    const int i = c0 + lane;
    const bool live = i < n_win;
    const uint32_t act = __ballot_sync(RB_FULL_MASK, live);
    if (live) {
      const uint2 e = w[i];
      const uint32_t peers = __match_any_sync(act, e.x);
      const int leader = __ffs(peers) - 1;
      int base = 0;
      if (lane == leader) base = atomicAdd(&start[e.x], __popc(peers));
      base = __shfl_sync(peers, base, leader);
      const int at = base + __popc(peers & lt);
      const int64_t id = a.pos != nullptr ? a.pos[static_cast<int64_t>(b) * a.L + e.y] : static_cast<int64_t>(e.y);
      ids[at] = id;
      sc[at] = static_cast<float>(bits - 2 * static_cast<int>(e.x));
    }
    __syncwarp();
  }
  for (int i = n_win + lane; i < a.k; i += 32) {
    ids[i] = -1;
    sc[i] = -INFINITY;
  }
}

int query_group(int B, int R, bool indirect) {
  if (indirect) return 1;  // each row ranks its own candidates
  return std::max(1, std::min({B, 32, 10240 / R}));  // histograms within 40 KB of shared memory
}

struct HamSelLayout {
  size_t hist, thr, bcnt, boff, win, total;
};

HamSelLayout ham_sel_layout(int B, int L, int W, int k) {
  HamSelLayout l{};
  const int64_t R = 64 * static_cast<int64_t>(W) + 1;
  const int64_t nblk = (static_cast<int64_t>(L) + kHsBlock - 1) / kHsBlock;
  size_t o = 0;
  l.hist = o;
  o += align_up(static_cast<size_t>(B) * R * 4, 256);
  l.thr = o;
  o += align_up(static_cast<size_t>(B) * 16, 256);
  l.bcnt = o;
  o += align_up(static_cast<size_t>(B) * nblk * 8, 256);
  l.boff = o;
  o += align_up(static_cast<size_t>(B) * nblk * 8, 256);
  l.win = o;
  o += align_up(static_cast<size_t>(B) * k * 8, 256);
  l.total = o;
  return l;
}

}  // namespace

size_t ham_select_ws_bytes(int B, int L, int W, int k) { return ham_sel_layout(B, L, W, k).total; }

int ham_select_topk(const uint64_t* qbits, const uint64_t* items, int N, int W, const int64_t* pos, int P,
                    const int64_t* counts, int B, int k, int64_t* out_ids, float* out_scores, void* ws,
                    size_t ws_bytes, cudaStream_t s) {
  const int L = pos != nullptr ? P : N;
  const HamSelLayout l = ham_sel_layout(B, L, W, k);
  if (ws == nullptr || ws_bytes < l.total) {
    set_last_error("hamming select: workspace too small");
    return RB_ERR_WORKSPACE;
  }
  if (B == 0 || k == 0) return RB_OK;
  uint8_t* w8 = static_cast<uint8_t*>(ws);
  HamSel a{qbits, items, pos, counts, B, N, W, L, k, 64 * W + 1, (L + kHsBlock - 1) / kHsBlock,
           reinterpret_cast<int*>(w8 + l.hist), reinterpret_cast<int*>(w8 + l.thr),
           reinterpret_cast<int*>(w8 + l.bcnt), reinterpret_cast<int*>(w8 + l.boff),
           reinterpret_cast<uint2*>(w8 + l.win)};
  if (cudaMemsetAsync(a.hist, 0, static_cast<size_t>(B) * a.R * 4, s) != cudaSuccess) {
    set_last_error("hamming select: memset failed");
    return RB_ERR_CUDA;
  }
  const int qg = query_group(B, a.R, pos != nullptr);
  const dim3 grid(std::max(a.nblk, 1), (B + qg - 1) / qg);
  const size_t q_bytes = static_cast<size_t>(qg) * W * 8;
  if (a.nblk > 0) {
    ham_hist_kernel<<<grid, kHsThreads, align_up(static_cast<size_t>(qg) * a.R * 4, 16) + q_bytes, s>>>(a, qg);
  }
  ham_threshold_kernel<<<(B + 127) / 128, 128, 0, s>>>(a);
  if (a.nblk > 0) {
    ham_block_kernel<false><<<grid, kHsThreads, q_bytes, s>>>(a, qg);
    ham_scan_kernel<<<B, 1024, 0, s>>>(a);
    ham_block_kernel<true><<<grid, kHsThreads, q_bytes, s>>>(a, qg);
  }
  ham_order_kernel<<<B, 32, static_cast<size_t>(a.R) * 4, s>>>(a, out_ids, out_scores);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

}  // namespace rb
