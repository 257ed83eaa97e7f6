// inst_f16.cu — kernel instantiations for A/B element type f16 (split per dtype so
// the build compiles them in parallel).
#include "gemm_launch.cuh"

namespace b200 {
B200_DEFINE_DISPATCH(launch_f16, DT_F16)
}  // namespace b200
