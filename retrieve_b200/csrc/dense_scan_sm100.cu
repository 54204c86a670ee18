// Fused dense scoring + exact top-k for sm_100a (B200): planning and dispatch.
//
// One persistent CTA per SM. A task is (query group, item split): the CTA
// holds NG x 128 queries resident in shared memory (TMA, 128-byte swizzle) and
// streams its split's item tiles (128 items each) through a STAGES-deep TMA
// ring. One elected thread issues tcgen05.mma (M = 128 queries, N = 128 items,
// K = the embedding dim) into a double-buffered TMEM accumulator; the epilogue
// warps read their query row out of TMEM (thread = query, 32 columns at a
// time), drop every 32-item chunk whose max is below the query's threshold and
// append the rest to the query's candidate list (rb_select.cuh). No [B, N]
// score matrix ever reaches HBM.
//
// Warp roles (NG = 2: 320 threads):
//   warp 0      TMA producer (queries once per task, item tiles per stage)
//   warp 1      TMEM allocator + MMA issuer
//   warps 2..   epilogue, 4 warps per query group (TMEM lane quadrant = warp % 4)
//
// Reference semantics replaced: PostfilterKNN.score + masked_topk
// (retrieve/src/retrieve/modules/knn.py:62-76, functional.py:57-85), i.e.
// torch.mm(q_fp16, E_t, out_dtype=fp32) followed by torch.topk, with ties broken
// toward the lower item id.
#include "dense_scan_kernels.cuh"

#include <atomic>
#include <mutex>

namespace rb {

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) == cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D K-major tensor map: rows x cols elements, box box_rows x 128 bytes, 128-B swizzle.
bool make_tmap_2d(CUtensorMap* map, const void* base, int elem, uint64_t rows, uint64_t cols, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const int eb = (elem == 2 || elem == 4) ? 1 : 2;
  CUtensorMapDataType dt = (elem == 2 || elem == 4) ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                           : (elem == 1)              ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * eb};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / eb), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace rb

// ---------------------------------------------------------------------------
// Scan-plan shared by the dense entry points.
// ---------------------------------------------------------------------------
namespace rb {

int list_cap(int k) {
  // room for k survivors + one 128-item tile of appends; multiple of 32
  return ((k + 128) + 31) / 32 * 32;
}

// Entries per lane of the register-resident list compaction for a list of cap.
static int dense_epl(int cap) { return cap <= 256 ? 8 : (cap <= 512 ? 16 : 40); }

// SMs of the current device, looked up once per device ordinal (thread-safe).
int num_sms() {
  static std::atomic<int> cached[kMaxCachedDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxCachedDevices) {
    cudaGetLastError();
    dev = -1;
  }
  if (dev >= 0) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 0;
  if (dev < 0 || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = 148;
  }
  if (dev >= 0) cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

void dense_plan(int B, int N, int k, int row_bytes, DensePlan& pl, int64_t n_total, bool scaled) {
  (void)scaled;  // the plan is the same for every element type
  // B > 128: 2-SM kernel, 256 queries per group, 1 or 2 groups per CTA pair
  // (one for 512-byte rows, whose operand tiles fill shared memory, and for
  // lists past 512 entries, whose compaction needs the registers of a 6-warp
  // CTA). The int8 dequant epilogue runs faster with two groups despite its
  // spills: the epilogue's issue rate, not spilling, bounds it.
  pl.two_sm = B > kQTile;
  if (pl.two_sm) {
    pl.ng = (B <= 2 * kQTile || row_bytes > 256 || list_cap(k) > 512) ? 1 : 2;
    pl.n_qsg = (B + pl.ng * 2 * kQTile - 1) / (pl.ng * 2 * kQTile);
    pl.n_splits = std::max(1, dense_max_pairs() / pl.n_qsg);
    pl.n_lists = pl.n_splits;
  } else {
    pl.ng = 1;
    pl.n_qsg = 1;
    pl.n_splits = num_sms();
    pl.n_lists = pl.n_splits;
  }
  pl.cap = list_cap(k);
  pl.tiles = (N + kTileItems - 1) / kTileItems;
  // Optional sampling pass over every s-th tile: it records the max score of each sampled
  // tile; the k-th largest tile max is a lower bound on the k-th best score of the corpus
  // (k distinct items reach it) and seeds the full pass. That bound sits near rank k * s of
  // the corpus, so the full pass appends about k * s candidates per query: s is the sparsest
  // stride (at most kSampleStride) that keeps those at no more than 0.1 per query row and
  // 128-item tile (over a corpus of n_total items: the union of every shard's sample when the
  // seed is shared) and still samples at least 4k tiles.
  pl.sample_stride = 0;
  const int64_t n_scale = std::max<int64_t>(n_total, N);
  for (int s = kSampleStride; s >= 1; s >>= 1) {
    const int64_t sampled = (pl.tiles + s - 1) / s;
    const bool dense_enough = static_cast<double>(k) * s * kTileItems <= 0.1 * static_cast<double>(n_scale);
    if (sampled >= 4 * static_cast<int64_t>(k) && (dense_enough || s == 1)) {
      pl.sample_stride = s;
      break;
    }
  }
}

// Values per query row of the sampling pass: one per sampled tile.
size_t dense_chunk_stride(const DensePlan& pl) {
  if (pl.sample_stride == 0) return 0;
  return static_cast<size_t>((pl.tiles + pl.sample_stride - 1) / pl.sample_stride);
}

size_t dense_workspace_bytes(int B, int N, int k, int row_bytes, bool scaled) {
  DensePlan pl;
  dense_plan(B, N, k, row_bytes, pl, N, scaled);
  size_t lists = static_cast<size_t>(B) * pl.n_lists * pl.cap * sizeof(uint2);
  size_t counts = static_cast<size_t>(B) * pl.n_lists * sizeof(int);
  // seeds [B] | safe seeds [B] | row flags [B] | query-group flags (at most B / 128 + 1)
  size_t th = (4 * static_cast<size_t>(B) + 64) * sizeof(float);
  size_t cm = static_cast<size_t>(B) * dense_chunk_stride(pl) * sizeof(float);
  // the chunk maxima are dead once the seed is known: they share the list space
  return align_up(std::max(lists, cm), 256) + align_up(counts, 256) + align_up(th, 256) + dense_spec_ws_bytes(k) +
         256;
}

size_t dense_spec_ws_bytes(int k) {
  const size_t r = kSpecRows;
  return align_up(r * 512, 256) + align_up(r * kMaxTerms * sizeof(PredTerm), 256) +
         align_up(r * static_cast<size_t>(k) * sizeof(int64_t), 256) +
         align_up(r * static_cast<size_t>(k) * sizeof(float), 256) + 5 * align_up(r * sizeof(int), 256) + 256;
}

int dense_scan_pass(int mode, int elem, const void* q, const void* x, int B, int N, int D, const DensePlan& pl,
                    int k, const float* seed, uint2* lists, int* counts, float* chunk_max, int* err,
                    cudaStream_t stream, const float* q_scale, const float* x_scale, const FilterArgs* filter,
                    const int* qsg_live) {
  DenseScanParams prm;
  std::memset(&prm, 0, sizeof(prm));
  const bool filtered = filter != nullptr && filter->mode != kFilterNone;
  if (filtered) prm.filter = *filter;
  prm.q_scale = q_scale;
  prm.x_scale = x_scale;
  const int eb = (elem == 2 || elem == 4) ? 1 : 2;
  const int row_bytes = D * eb;
  const int item_box = pl.two_sm ? kHalfItems : kTileItems;
  if (!make_tmap_2d(&prm.tmap_q, q, elem, static_cast<uint64_t>(B), static_cast<uint64_t>(D), kQTile) ||
      !make_tmap_2d(&prm.tmap_x, x, elem, static_cast<uint64_t>(N), static_cast<uint64_t>(D), item_box)) {
    set_last_error("cuTensorMapEncodeTiled failed (alignment or driver entry point)");
    return RB_ERR_CUDA;
  }
  const int stride = (mode == 1) ? pl.sample_stride : 1;
  prm.seed = seed;
  prm.lists = lists;
  prm.counts = counts;
  prm.err = err;
  prm.chunk_max = chunk_max;
  prm.chunk_stride = static_cast<int>(dense_chunk_stride(pl));
  prm.B = B;
  prm.N = N;
  prm.n_qsg = pl.n_qsg;
  prm.n_splits = pl.n_splits;
  prm.tile_stride = stride;
  prm.tile_offset = 0;
  prm.pass_tiles = (pl.tiles + stride - 1) / stride;
  prm.k = k;
  prm.cap = pl.cap;
  prm.qsg_live = qsg_live;
  if (filtered && pl.two_sm) {
    // The 2-SM filtered kernel streams each tile's Bloom slices and (rows of at most 8 cells,
    // a whole number of 16-byte units, 16-byte aligned) attribute rows through a shared-memory
    // ring beside the item tiles; other rows are read from global memory item by item.
    const FilterArgs& f = prm.filter;
    const bool sliced = f.slices != nullptr && (f.mode == kFilterBloom || f.mode == kFilterBloomRecheck);
    const int ca = f.C * f.A;
    const bool rows = f.attrs != nullptr && (f.mode == kFilterExact || f.mode == kFilterBloomRecheck) && ca >= 1 &&
                      ca <= 8 && ca % 2 == 0 && (reinterpret_cast<uintptr_t>(f.attrs) & 15u) == 0;
    prm.ring = (sliced ? 1 : 0) | (rows ? 2 : 0);
  }
  const int n_tasks = pl.n_qsg * pl.n_splits;
  cudaError_t e = cudaSuccess;
  const int kb = row_bytes / 128;
  const int epl = dense_epl(pl.cap);
  const int grid = pl.two_sm ? std::min(n_tasks, dense_max_pairs()) : std::min(n_tasks, num_sms());
  bool handled = false;
  switch (elem) {
    case 0: handled = dense_launch_e0(pl.two_sm, mode, kb, pl.ng, filtered, epl, prm, grid, stream, e); break;
    case 1: handled = dense_launch_e1(pl.two_sm, mode, kb, pl.ng, filtered, epl, prm, grid, stream, e); break;
    case 2: handled = dense_launch_e2(pl.two_sm, mode, kb, pl.ng, filtered, epl, prm, grid, stream, e); break;
    case 4: handled = dense_launch_e4(pl.two_sm, mode, kb, pl.ng, filtered, epl, prm, grid, stream, e); break;
    default: break;
  }
  if (!handled) {
    set_last_error("dense scan: unsupported dtype / row width");
    return RB_ERR_UNSUPPORTED;
  }
  if (e != cudaSuccess) {
    char msg[256];
    std::snprintf(msg, sizeof(msg), "%s (dense scan launch: pass %d, %s kernel, %d K-blocks, %d query tiles%s)",
                  cudaGetErrorString(e), mode, pl.two_sm ? "2-SM" : "1-SM", kb, pl.ng, filtered ? ", filtered" : "");
    set_last_error(msg);
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

}  // namespace rb
