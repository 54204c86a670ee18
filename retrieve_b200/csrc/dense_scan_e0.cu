// Dense scan variants for element type 0: fp16.
#include "dense_scan_kernels.cuh"

namespace rb {

bool dense_launch_e0(bool two_sm, int mode, int kb, int ng, bool filtered, int epl, const DenseScanParams& prm,
                     int grid, cudaStream_t stream, cudaError_t& e) {
#define RB_V2(KB, NG, ST, F)                                                            \
  if (two_sm && kb == KB && ng == NG && filtered == F) {                                \
    e = launch_2sm_variant<0, KB, NG, ST, F>(mode, epl, prm, grid, stream);              \
    return true;                                                                        \
  }
#define RB_V1(KB, NG, ST, F)                                                            \
  if (!two_sm && kb == KB && ng == NG && filtered == F) {                               \
    e = launch_1sm_variant<0, KB, NG, ST, F>(mode, epl, prm, grid, stream);              \
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
