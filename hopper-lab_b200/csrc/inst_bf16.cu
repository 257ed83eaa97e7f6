// inst_bf16.cu — kernel instantiations for A/B element type bf16 (split per dtype so
// the build compiles them in parallel).
#include "gemm_launch.cuh"

namespace b200 {
B200_DEFINE_DISPATCH(launch_bf16, DT_BF16)
}  // namespace b200
