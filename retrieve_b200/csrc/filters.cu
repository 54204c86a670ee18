// The exact clause filter and the single-query GEMV.
//
// Clause predicate (retrieve/src/retrieve/functional.py:173-185
// `clause_subset_match`; Triton `clause_pass`, ops/triton/common.py:48-80):
// item n passes query b iff for every clause c with q[b, c] != -1,
// (any_a attrs[n, c, a] == q[b, c]) XOR reverse[c]. An inactive clause
// (q == -1) passes. Attrs are int64 [N, C, A] with -1 padding, queries int64
// [B, C], reverse flags bool [C].
//
// gemv_scores (ops/triton/gemv_scores.py:19-43): one fp16 query [1, D] against
// the fp16 table E_t [D, N]: out[n] = fma(q[D-1], E_t[D-1, n], ... fma(q[0],
// E_t[0, n], 0)) in fp32, k = 0 .. D-1 in order.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>

#include "rb_capi_internal.h"
#include "rb_common.cuh"

namespace rb {

constexpr int kFilterQB = 8;  // queries per CTA row of the clause kernels

struct ClauseArgs {
  const int64_t* attrs;    // [N, C, A]
  const uint8_t* reverse;  // [C]
  const int64_t* qattrs;   // [B, C]
  int N, C, A, B;
};

// Evaluates the predicate of item n for queries b0 .. b0+nq-1 (query attrs and
// reverse flags staged in shared memory). Bit i of the result is query b0 + i.
__device__ __forceinline__ uint32_t clause_bits(const ClauseArgs& a, const int64_t* __restrict__ sq,
                                                const uint8_t* __restrict__ srev, int nq, int64_t n) {
  uint32_t bits = (nq >= 32) ? 0xffffffffu : ((1u << nq) - 1u);
  const int64_t* row = a.attrs + n * a.C * a.A;
  for (int c = 0; c < a.C; ++c) {
    const int64_t* cell = row + c * a.A;
    for (int i = 0; i < nq; ++i) {
      const int64_t qv = sq[i * a.C + c];
      if (qv == -1) continue;
      bool m = false;
      for (int j = 0; j < a.A; ++j) m |= (cell[j] == qv);
      if (m == static_cast<bool>(srev[c])) bits &= ~(1u << i);
    }
  }
  return bits;
}

template <bool SCORES>
__global__ void __launch_bounds__(256) clause_mask_kernel(ClauseArgs a, const float* __restrict__ scores,
                                                          void* __restrict__ out) {
  extern __shared__ int64_t sq[];  // [kFilterQB, C] then reverse flags
  uint8_t* srev = reinterpret_cast<uint8_t*>(sq + kFilterQB * a.C);
  const int b0 = blockIdx.y * kFilterQB;
  const int nq = min(kFilterQB, a.B - b0);
  for (int i = threadIdx.x; i < nq * a.C; i += blockDim.x) sq[i] = a.qattrs[static_cast<int64_t>(b0) * a.C + i];
  for (int i = threadIdx.x; i < a.C; i += blockDim.x) srev[i] = a.reverse[i];
  __syncthreads();
  for (int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; n < a.N;
       n += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t bits = clause_bits(a, sq, srev, nq, n);
    for (int i = 0; i < nq; ++i) {
      const size_t o = static_cast<size_t>(b0 + i) * a.N + n;
      const bool pass = (bits >> i) & 1u;
      if constexpr (SCORES)
        static_cast<float*>(out)[o] = pass ? scores[o] : -INFINITY;
      else
        static_cast<uint8_t*>(out)[o] = pass ? 1 : 0;
    }
  }
}

// clause_compact phase 1: passing items per (row, tile).
constexpr int kCompactTile = 1024;

__global__ void __launch_bounds__(256) clause_count_kernel(ClauseArgs a, int n_tiles, int* __restrict__ tile_counts) {
  extern __shared__ int64_t sq[];
  uint8_t* srev = reinterpret_cast<uint8_t*>(sq + kFilterQB * a.C);
  __shared__ int warp_sum[kFilterQB][8];
  const int b0 = blockIdx.y * kFilterQB;
  const int nq = min(kFilterQB, a.B - b0);
  for (int i = threadIdx.x; i < nq * a.C; i += blockDim.x) sq[i] = a.qattrs[static_cast<int64_t>(b0) * a.C + i];
  for (int i = threadIdx.x; i < a.C; i += blockDim.x) srev[i] = a.reverse[i];
  __syncthreads();
  const int t = blockIdx.x;
  int cnt[kFilterQB] = {0};
  for (int j = threadIdx.x; j < kCompactTile; j += blockDim.x) {
    const int64_t n = static_cast<int64_t>(t) * kCompactTile + j;
    if (n >= a.N) break;
    const uint32_t bits = clause_bits(a, sq, srev, nq, n);
#pragma unroll
    for (int i = 0; i < kFilterQB; ++i) cnt[i] += (bits >> i) & 1u;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < kFilterQB; ++i) {
    int v = cnt[i];
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(RB_FULL_MASK, v, off);
    if (lane == 0) warp_sum[i][warp] = v;
  }
  __syncthreads();
  if (threadIdx.x < nq) {
    int s = 0;
    for (int w = 0; w < 8; ++w) s += warp_sum[threadIdx.x][w];
    tile_counts[static_cast<size_t>(b0 + threadIdx.x) * n_tiles + t] = s;
  }
}

// clause_compact phase 2: per row, exclusive scan of the tile counts (in place)
// and the row total.
__global__ void __launch_bounds__(1024) clause_scan_kernel(int* __restrict__ tile_counts, int n_tiles,
                                                           int64_t* __restrict__ counts) {
  __shared__ int warp_tot[32];
  __shared__ int carry;
  const int b = blockIdx.x;
  int* row = tile_counts + static_cast<size_t>(b) * n_tiles;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < n_tiles; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int v = (i < n_tiles) ? row[i] : 0;
    int incl = v;
    for (int off = 1; off < 32; off <<= 1) {
      const int u = __shfl_up_sync(RB_FULL_MASK, incl, off);
      if (lane >= off) incl += u;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = (lane < static_cast<int>(blockDim.x >> 5)) ? warp_tot[lane] : 0;
      for (int off = 1; off < 32; off <<= 1) {
        const int u = __shfl_up_sync(RB_FULL_MASK, w, off);
        if (lane >= off) w += u;
      }
      warp_tot[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int before = carry + (warp > 0 ? warp_tot[warp - 1] : 0) + incl - v;
    if (i < n_tiles) row[i] = before;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = before + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) counts[b] = carry;
}

// clause_compact phase 3: the passing ids of each (row, tile), in ascending
// order, at the tile's scanned offset. One query per CTA row here (ranks need
// a block-wide prefix per query).
__global__ void __launch_bounds__(256) clause_scatter_kernel(ClauseArgs a, int n_tiles,
                                                             const int* __restrict__ tile_offsets,
                                                             int64_t* __restrict__ out) {
  extern __shared__ int64_t sq[];
  uint8_t* srev = reinterpret_cast<uint8_t*>(sq + a.C);
  __shared__ int warp_tot[8];
  __shared__ int base_s;
  const int b = blockIdx.y;
  for (int i = threadIdx.x; i < a.C; i += blockDim.x) {
    sq[i] = a.qattrs[static_cast<int64_t>(b) * a.C + i];
    srev[i] = a.reverse[i];
  }
  const int t = blockIdx.x;
  if (threadIdx.x == 0) base_s = tile_offsets[static_cast<size_t>(b) * n_tiles + t];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t* orow = out + static_cast<size_t>(b) * a.N;
  for (int j0 = 0; j0 < kCompactTile; j0 += blockDim.x) {
    const int64_t n = static_cast<int64_t>(t) * kCompactTile + j0 + threadIdx.x;
    const bool pass = (n < a.N) && (clause_bits(a, sq, srev, 1, n) & 1u);
    const uint32_t bal = __ballot_sync(RB_FULL_MASK, pass);
    if (lane == 0) warp_tot[warp] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < 8; ++w) {
      before += (w < warp) ? warp_tot[w] : 0;
      total += warp_tot[w];
    }
    if (pass) orow[base_s + before + __popc(bal & lanemask_lt())] = n;
    __syncthreads();
    if (threadIdx.x == 0) base_s += total;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// gemv_scores
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gemv_vec8_kernel(const __half* __restrict__ q, const __half* __restrict__ et,
                                                        int D, int N, float* __restrict__ out) {
  extern __shared__ float sq_f[];
  for (int i = threadIdx.x; i < D; i += blockDim.x) sq_f[i] = __half2float(q[i]);
  __syncthreads();
  const int64_t n0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (n0 >= N) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int k = 0; k < D; ++k) {
    const uint4 v = *reinterpret_cast<const uint4*>(et + static_cast<int64_t>(k) * N + n0);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
    const float qk = sq_f[k];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      acc[2 * i] = fmaf(qk, f.x, acc[2 * i]);
      acc[2 * i + 1] = fmaf(qk, f.y, acc[2 * i + 1]);
    }
  }
  float4* o = reinterpret_cast<float4*>(out + n0);
  o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

__global__ void __launch_bounds__(256) gemv_scalar_kernel(const __half* __restrict__ q,
                                                          const __half* __restrict__ et, int D, int N,
                                                          float* __restrict__ out) {
  extern __shared__ float sq_f[];
  for (int i = threadIdx.x; i < D; i += blockDim.x) sq_f[i] = __half2float(q[i]);
  __syncthreads();
  const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float acc = 0.f;
  for (int k = 0; k < D; ++k) acc = fmaf(sq_f[k], __half2float(et[static_cast<int64_t>(k) * N + n]), acc);
  out[n] = acc;
}

static int launch_check(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  (void)what;
  return RB_OK;
}

static int clause_grid_x(int N) { return std::max(1, std::min((N + 255) / 256, 4 * num_sms())); }

}  // namespace rb

using namespace rb;

extern "C" {

int rb_clause_mask(const int64_t* item_attrs, int N, int C, int A, const uint8_t* is_reverse,
                   const int64_t* query_attrs, int B, const float* scores, void* out, void* stream) {
  if (N < 0 || C < 0 || A < 0 || B < 0) {
    set_last_error("clause_mask: negative size");
    return RB_ERR_INVALID_ARG;
  }
  if (B == 0 || N == 0) return RB_OK;
  ClauseArgs a{item_attrs, is_reverse, query_attrs, N, C, A, B};
  const dim3 grid(clause_grid_x(N), (B + kFilterQB - 1) / kFilterQB);
  const size_t smem = kFilterQB * static_cast<size_t>(C) * sizeof(int64_t) + C + 8;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (scores)
    clause_mask_kernel<true><<<grid, 256, smem, s>>>(a, scores, out);
  else
    clause_mask_kernel<false><<<grid, 256, smem, s>>>(a, nullptr, out);
  return launch_check("clause_mask");
}

int rb_clause_compact_workspace_size(int B, int N, size_t* bytes) {
  if (bytes == nullptr || B < 0 || N < 0) {
    set_last_error("clause_compact_workspace_size: bad arguments");
    return RB_ERR_INVALID_ARG;
  }
  const size_t tiles = (static_cast<size_t>(N) + kCompactTile - 1) / kCompactTile;
  *bytes = align_up(static_cast<size_t>(B) * std::max<size_t>(tiles, 1) * sizeof(int), 256);
  return RB_OK;
}

int rb_clause_compact(const int64_t* item_attrs, int N, int C, int A, const uint8_t* is_reverse,
                      const int64_t* query_attrs, int B, int64_t* out_ids, int64_t* out_counts, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (N < 0 || C < 0 || A < 0 || B < 0) {
    set_last_error("clause_compact: negative size");
    return RB_ERR_INVALID_ARG;
  }
  if (B == 0) return RB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (N == 0) {
    return cudaMemsetAsync(out_counts, 0, static_cast<size_t>(B) * sizeof(int64_t), s) == cudaSuccess
               ? RB_OK
               : (set_last_error("memset failed"), RB_ERR_CUDA);
  }
  size_t need = 0;
  rb_clause_compact_workspace_size(B, N, &need);
  if (workspace == nullptr || workspace_bytes < need) {
    set_last_error("clause_compact: workspace too small");
    return RB_ERR_WORKSPACE;
  }
  const int n_tiles = (N + kCompactTile - 1) / kCompactTile;
  int* tiles = static_cast<int*>(workspace);
  ClauseArgs a{item_attrs, is_reverse, query_attrs, N, C, A, B};
  const size_t smem8 = kFilterQB * static_cast<size_t>(C) * sizeof(int64_t) + C + 8;
  clause_count_kernel<<<dim3(n_tiles, (B + kFilterQB - 1) / kFilterQB), 256, smem8, s>>>(a, n_tiles, tiles);
  int rc = launch_check("clause_count");
  if (rc != RB_OK) return rc;
  clause_scan_kernel<<<B, 1024, 0, s>>>(tiles, n_tiles, out_counts);
  rc = launch_check("clause_scan");
  if (rc != RB_OK) return rc;
  const size_t smem1 = static_cast<size_t>(C) * sizeof(int64_t) + C + 8;
  clause_scatter_kernel<<<dim3(n_tiles, B), 256, smem1, s>>>(a, n_tiles, tiles, out_ids);
  return launch_check("clause_scatter");
}

int rb_gemv_scores(const void* query, const void* items_t, int D, int N, float* out, void* stream) {
  if (D <= 0 || N < 0) {
    set_last_error("gemv_scores: bad D or N");
    return RB_ERR_INVALID_ARG;
  }
  if (N == 0) return RB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = static_cast<size_t>(D) * sizeof(float);
  const bool vec = (N % 8 == 0) && ((reinterpret_cast<uintptr_t>(items_t) & 15u) == 0) &&
                   ((reinterpret_cast<uintptr_t>(out) & 15u) == 0);
  if (vec) {
    const int threads = (N / 8 + 255) / 256;
    gemv_vec8_kernel<<<threads, 256, smem, s>>>(static_cast<const __half*>(query),
                                                static_cast<const __half*>(items_t), D, N, out);
  } else {
    gemv_scalar_kernel<<<(N + 255) / 256, 256, smem, s>>>(static_cast<const __half*>(query),
                                                          static_cast<const __half*>(items_t), D, N, out);
  }
  return launch_check("gemv_scores");
}

}  // extern "C"
