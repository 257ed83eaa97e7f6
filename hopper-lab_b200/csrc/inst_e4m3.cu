// inst_e4m3.cu — kernel instantiations for A/B element type e4m3 (split per dtype so
// the build compiles them in parallel).
#include "gemm_launch.cuh"

namespace b200 {
B200_DEFINE_DISPATCH(launch_e4m3, DT_E4M3)
}  // namespace b200
