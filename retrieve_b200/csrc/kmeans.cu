// The centroid update of the IVF build's k-means (retrieve/src/retrieve/indexing/kmeans.py:40-60,
// 98-119): per cluster the fp64 sum of its member rows and the member count. The reference
// reduces with one fp64 one-hot GEMM per row chunk (n_lists x chunk x D multiply-adds, almost
// all of them by zero) so that the order of the additions is fixed by the shapes; here the
// order is fixed by a stable counting sort instead, and each cluster's rows are added in
// increasing row order in fp64: N x D additions, the same per-cluster sums up to the rounding of
// fp64 additions (exact when the fp64 sums are), and bit-for-bit reproducible run to run.
//
//  1. km_walk_kernel<false>: the rows cut into chunks; one warp per chunk counts its rows per
//     cluster into table[cluster][chunk] (the warp owns the chunk's column: no atomics).
//  2. scan_tiles / scan_totals / scan_add: exclusive scan of the table in cluster-major order,
//     so table[c][k] becomes the first output slot of cluster c's rows from chunk k.
//  3. km_walk_kernel<true>: the warps walk their chunks again in row order and write each row
//     index at its slot (ranks within a warp batch by lane order): a stable sort by cluster.
//  4. km_sum_kernel: one CTA per cluster, a thread per dimension, the cluster's rows added in
//     order in fp64.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "rb_capi_internal.h"
#include "rb_common.cuh"

namespace rb {
namespace {

constexpr int kWarpsPerBlock = 8;
constexpr int kScanThreads = 1024;
constexpr int kScanTile = 2 * kScanThreads;
constexpr int kSumThreads = 256;
constexpr int64_t kMaxTableEntries = int64_t{1} << 24;  // (cluster, chunk) counters: 128 MiB of int64

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

struct Plan {
  int64_t chunk;     // rows per warp chunk (a multiple of 32)
  int64_t n_chunks;  // ceil(N / chunk)
  int64_t entries;   // n_lists * n_chunks
  int64_t tiles;     // scan tiles of the table
};

Plan plan_for(int64_t N, int64_t n_lists) {
  Plan p;
  const int64_t min_chunk = (N * n_lists + kMaxTableEntries - 1) / kMaxTableEntries;
  p.chunk = std::max<int64_t>(1024, (min_chunk + 31) / 32 * 32);
  p.n_chunks = std::max<int64_t>(1, (N + p.chunk - 1) / p.chunk);
  p.entries = n_lists * p.n_chunks;
  p.tiles = (p.entries + kScanTile - 1) / kScanTile;
  return p;
}

// Steps 1 and 3: each warp walks its chunk in batches of 32 rows; lanes holding the same cluster
// form a group whose lowest lane owns the group's counter update.
template <bool SCATTER>
__global__ void __launch_bounds__(32 * kWarpsPerBlock) km_walk_kernel(const int64_t* __restrict__ assign, int64_t N,
                                                                       int64_t n_lists, int64_t chunk,
                                                                       int64_t n_chunks, int64_t* __restrict__ table,
                                                                       int64_t* __restrict__ order) {
  const int lane = threadIdx.x & 31;
  const int64_t w = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  if (w >= n_chunks) return;  // warp-uniform
  const int64_t begin = w * chunk, end = min(N, begin + chunk);
  for (int64_t base = begin; base < end; base += 32) {
    const int64_t row = base + lane;
    int64_t c = row < end ? assign[row] : -1;
    if (c < 0 || c >= n_lists) c = -1;  // rows outside any cluster are left out
    const uint32_t group = __match_any_sync(RB_FULL_MASK, static_cast<unsigned long long>(c));
    const int leader = __ffs(group) - 1;
    int64_t* counter = c >= 0 ? table + c * n_chunks + w : nullptr;
    if constexpr (SCATTER) {
      if (c >= 0) order[*counter + __popc(group & lanemask_lt())] = row;
      __syncwarp();
    }
    if (c >= 0 && lane == leader) *counter += __popc(group);
    __syncwarp();
  }
}

// Exclusive scan of n int64 values in place: per-tile scans with tile totals, a one-CTA scan of
// the totals, then the totals' prefixes added back.
__device__ int64_t block_exclusive_scan(int64_t v, int64_t* part, int64_t& total) {
  const int tid = threadIdx.x;
  part[tid] = v;
  __syncthreads();
  for (int off = 1; off < kScanThreads; off <<= 1) {
    const int64_t x = tid >= off ? part[tid - off] : 0;
    __syncthreads();
    part[tid] += x;
    __syncthreads();
  }
  total = part[kScanThreads - 1];
  const int64_t incl = part[tid];
  __syncthreads();
  return incl - v;
}

__global__ void __launch_bounds__(kScanThreads) scan_tiles_kernel(int64_t* __restrict__ a, int64_t n,
                                                                   int64_t* __restrict__ totals) {
  __shared__ int64_t part[kScanThreads];
  const int64_t i0 = static_cast<int64_t>(blockIdx.x) * kScanTile + 2 * threadIdx.x;
  const int64_t x0 = i0 < n ? a[i0] : 0, x1 = i0 + 1 < n ? a[i0 + 1] : 0;
  int64_t total;
  const int64_t ex = block_exclusive_scan(x0 + x1, part, total);
  if (i0 < n) a[i0] = ex;
  if (i0 + 1 < n) a[i0 + 1] = ex + x0;
  if (threadIdx.x == 0) totals[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kScanThreads) scan_totals_kernel(int64_t* __restrict__ totals, int64_t n) {
  __shared__ int64_t part[kScanThreads];
  const int64_t per = (n + kScanThreads - 1) / kScanThreads;
  const int64_t i0 = min(n, threadIdx.x * per), i1 = min(n, i0 + per);
  int64_t run = 0;
  for (int64_t i = i0; i < i1; ++i) run += totals[i];
  int64_t total;
  int64_t acc = block_exclusive_scan(run, part, total);
  for (int64_t i = i0; i < i1; ++i) {
    const int64_t v = totals[i];
    totals[i] = acc;
    acc += v;
  }
}

__global__ void __launch_bounds__(kScanThreads) scan_add_kernel(int64_t* __restrict__ a, int64_t n,
                                                                 const int64_t* __restrict__ totals) {
  const int64_t add = totals[blockIdx.x];
  const int64_t i0 = static_cast<int64_t>(blockIdx.x) * kScanTile + 2 * threadIdx.x;
  if (i0 < n) a[i0] += add;
  if (i0 + 1 < n) a[i0 + 1] += add;
}

template <typename T>
__device__ __forceinline__ double to_f64(const T* x, int64_t i);
template <>
__device__ __forceinline__ double to_f64<float>(const float* x, int64_t i) { return static_cast<double>(x[i]); }
template <>
__device__ __forceinline__ double to_f64<__half>(const __half* x, int64_t i) {
  return static_cast<double>(__half2float(x[i]));
}
template <>
__device__ __forceinline__ double to_f64<__nv_bfloat16>(const __nv_bfloat16* x, int64_t i) {
  return static_cast<double>(__bfloat162float(x[i]));
}

// Step 4. The scatter has advanced every counter past its chunk's rows, so table[c][k] now
// holds the start of (c, k + 1) and table[c][n_chunks - 1] the end of cluster c: cluster c's
// rows are order[end(c - 1) .. end(c)), added in that order.
template <typename T>
__global__ void __launch_bounds__(kSumThreads) km_sum_kernel(const T* __restrict__ x, int D,
                                                              const int64_t* __restrict__ order,
                                                              const int64_t* __restrict__ table, int64_t n_chunks,
                                                              double* __restrict__ sums, int64_t* __restrict__ counts) {
  const int64_t c = blockIdx.x;
  const int64_t s0 = c == 0 ? 0 : table[c * n_chunks - 1];
  const int64_t s1 = table[(c + 1) * n_chunks - 1];
  if (threadIdx.x == 0) counts[c] = s1 - s0;
  for (int d0 = 0; d0 < D; d0 += kSumThreads) {
    const int d = d0 + threadIdx.x;
    double acc = 0.0;
    if (d < D)
      for (int64_t i = s0; i < s1; ++i) acc += to_f64(x, order[i] * D + d);
    if (d < D) sums[c * D + d] = acc;
  }
}

}  // namespace
}  // namespace rb

using namespace rb;

extern "C" {

int rb_kmeans_cluster_sums_workspace_size(int64_t N, int64_t n_lists, size_t* bytes) {
  if (bytes == nullptr || N < 0 || n_lists < 1 || n_lists > kMaxTableEntries) {
    set_last_error("kmeans_cluster_sums_workspace_size: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  const Plan p = plan_for(N, n_lists);
  *bytes = align_up(static_cast<size_t>(p.entries) * 8, 256) + align_up(static_cast<size_t>(p.tiles) * 8, 256) +
           align_up(static_cast<size_t>(std::max<int64_t>(N, 1)) * 8, 256);
  return RB_OK;
}

int rb_kmeans_cluster_sums(const void* embs, int dtype, int64_t N, int D, const int64_t* assignments,
                           int64_t n_lists, double* out_sums, int64_t* out_counts, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (N < 0 || D < 1 || n_lists < 1 || n_lists > kMaxTableEntries ||
      (N > 0 && (embs == nullptr || assignments == nullptr)) ||
      out_sums == nullptr || out_counts == nullptr) {
    set_last_error("kmeans_cluster_sums: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  if (dtype != RB_F32 && dtype != RB_F16 && dtype != RB_BF16) {
    set_last_error("kmeans_cluster_sums: embeddings must be fp32, fp16 or bf16");
    return RB_ERR_TYPE;
  }
  size_t need = 0;
  rb_kmeans_cluster_sums_workspace_size(N, n_lists, &need);
  if (workspace == nullptr || workspace_bytes < need) {
    set_last_error("kmeans_cluster_sums: workspace too small");
    return RB_ERR_WORKSPACE;
  }
  const Plan p = plan_for(N, n_lists);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int64_t* table = reinterpret_cast<int64_t*>(ws);
  ws += align_up(static_cast<size_t>(p.entries) * 8, 256);
  int64_t* totals = reinterpret_cast<int64_t*>(ws);
  ws += align_up(static_cast<size_t>(p.tiles) * 8, 256);
  int64_t* order = reinterpret_cast<int64_t*>(ws);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  cudaError_t e = cudaMemsetAsync(table, 0, static_cast<size_t>(p.entries) * 8, s);
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  const int walk_blocks = static_cast<int>((p.n_chunks + kWarpsPerBlock - 1) / kWarpsPerBlock);
  if (N > 0)
    km_walk_kernel<false><<<walk_blocks, 32 * kWarpsPerBlock, 0, s>>>(assignments, N, n_lists, p.chunk, p.n_chunks,
                                                                      table, order);
  scan_tiles_kernel<<<static_cast<unsigned>(p.tiles), kScanThreads, 0, s>>>(table, p.entries, totals);
  scan_totals_kernel<<<1, kScanThreads, 0, s>>>(totals, p.tiles);
  scan_add_kernel<<<static_cast<unsigned>(p.tiles), kScanThreads, 0, s>>>(table, p.entries, totals);
  int rc = launch_status();
  if (rc != RB_OK) return rc;
  if (N > 0)
    km_walk_kernel<true><<<walk_blocks, 32 * kWarpsPerBlock, 0, s>>>(assignments, N, n_lists, p.chunk, p.n_chunks,
                                                                     table, order);
  const unsigned grid = static_cast<unsigned>(n_lists);
  if (dtype == RB_F32)
    km_sum_kernel<float><<<grid, kSumThreads, 0, s>>>(static_cast<const float*>(embs), D, order, table, p.n_chunks,
                                                      out_sums, out_counts);
  else if (dtype == RB_F16)
    km_sum_kernel<__half><<<grid, kSumThreads, 0, s>>>(static_cast<const __half*>(embs), D, order, table,
                                                       p.n_chunks, out_sums, out_counts);
  else
    km_sum_kernel<__nv_bfloat16><<<grid, kSumThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(embs), D, order,
                                                              table, p.n_chunks, out_sums, out_counts);
  return launch_status();
}

}  // extern "C"
