// Dense scan variants for element type 1: bf16.
#include "dense_scan_kernels.cuh"

#include <atomic>

namespace rb {

// CTA pairs of the 2-SM kernel that fit on the current device at once, looked up once per
// device ordinal (thread-safe).
int dense_max_pairs() {
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
  const int sms = num_sms();
  using L = Dense2SmLayout<2, 2, 8>;
  auto kern = dense_scan_2sm_kernel<0, 1, 2, 2, 8, 16, false>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
  cfg.blockDim = dim3(64 + 128 * 2, 1, 1);
  cfg.dynamicSmemBytes = L::kTotal;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
    cudaGetLastError();
    clusters = sms / 2;
  }
  const int n = std::max(1, std::min(clusters, sms / 2));
  if (dev >= 0) cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

bool dense_launch_e1(bool two_sm, int mode, int kb, int ng, bool filtered, int epl, const DenseScanParams& prm,
                     int grid, cudaStream_t stream, cudaError_t& e) {
#define RB_V2(KB, NG, ST, F)                                                            \
  if (two_sm && kb == KB && ng == NG && filtered == F) {                                \
    e = launch_2sm_variant<1, KB, NG, ST, F>(mode, epl, prm, grid, stream);              \
    return true;                                                                        \
  }
#define RB_V1(KB, NG, ST, F)                                                            \
  if (!two_sm && kb == KB && ng == NG && filtered == F) {                               \
    e = launch_1sm_variant<1, KB, NG, ST, F>(mode, epl, prm, grid, stream);              \
    return true;                                                                        \
  }
  RB_V2(1, 1, 12, false)
  RB_V2(1, 2, 12, false)
  RB_V2(2, 1, 8, false)
  RB_V2(2, 2, 8, false)
  RB_V2(4, 1, 4, false)
  RB_V2(1, 1, 12, true)
  RB_V2(1, 2, 12, true)
  RB_V2(2, 1, 8, true)
  RB_V2(2, 2, 5, true)
  RB_V1(1, 1, 8, false)
  RB_V1(2, 1, 4, false)
  RB_V1(4, 1, 2, false)
  RB_V1(1, 1, 8, true)
  RB_V1(2, 1, 4, true)
#undef RB_V1
#undef RB_V2
  return false;
}

}  // namespace rb
