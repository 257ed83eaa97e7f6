// gemm_launch.cuh — launch wrapper shared by the per-dtype instantiation units.
#pragma once

#include <cuda_runtime.h>

#include "gemm_sm100.cuh"

namespace b200 {

struct LaunchPlan {
  const CUtensorMap* a;
  const CUtensorMap* b;
  const CUtensorMap* c;
  KParams kp;
  uint32_t grid;   // CTAs (a multiple of CG)
  uint32_t smem;   // dynamic shared memory bytes
  cudaStream_t stream;
};

template <int AB, int CD, int CG, int SCHED, int TN>
cudaError_t launch_gemm(const LaunchPlan& lp) {
  using Cfg = GemmCfg<AB, CD, CG, SCHED, TN>;
  auto kern = gemm_tcgen05_kernel<AB, CD, CG, SCHED, TN>;
  // The opt-in shared-memory size is a per-function, per-device attribute.
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(Cfg::MAX_SMEM));
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(lp.grid, 1, 1);
  cfg.blockDim = dim3(Cfg::NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = lp.smem;
  cfg.stream = lp.stream;
  cudaLaunchAttribute attr[2];
  // programmatic dependent launch: the kernel waits (griddepcontrol.wait) for the
  // previous kernel of the stream before touching global memory, so its launch and
  // set-up may overlap that kernel's tail (2048^3 back to back: 18.5 -> 16.5 us)
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (CG == 2) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  if (SCHED == SCHED_STREAMK) {
    // A split tile's last owner waits for the earlier owners' partial sums, so the
    // whole grid must be resident at once: clamp it to the clusters that fit.
    static int max_clusters[64] = {0};
    if (!max_clusters[dev]) {
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      if (e != cudaSuccess) return e;
      if (n < 1) return cudaErrorInvalidConfiguration;
      max_clusters[dev] = n;
    }
    if (cfg.gridDim.x > uint32_t(max_clusters[dev]) * CG) cfg.gridDim.x = uint32_t(max_clusters[dev]) * CG;
  }
  return cudaLaunchKernelEx(&cfg, kern, *lp.a, *lp.b, *lp.c, lp.kp);
}

// One dispatch entry per A/B type — defined in the instantiation units. Selects
// the instantiation for (C type, CTAs per tile, schedule, tile width).
cudaError_t launch_f16(int cd, int cg, int sched, int tn, const LaunchPlan& lp);
cudaError_t launch_bf16(int cd, int cg, int sched, int tn, const LaunchPlan& lp);
cudaError_t launch_e4m3(int cd, int cg, int sched, int tn, const LaunchPlan& lp);

#define B200_DISPATCH_CD(AB, CG, SCHED, TN)                                              \
  do {                                                                                   \
    if (cd == DT_F16) return launch_gemm<AB, DT_F16, CG, SCHED, TN>(lp);                 \
    if (cd == DT_BF16) return launch_gemm<AB, DT_BF16, CG, SCHED, TN>(lp);               \
    if (cd == DT_F32) return launch_gemm<AB, DT_F32, CG, SCHED, TN>(lp);                 \
  } while (0)

// Built: 1-CTA 128x256 (static, CLC); pairs 256x128 and 256x256 (static, CLC,
// stream-K) and 256x512 (static, CLC).
#define B200_DEFINE_DISPATCH(NAME, AB)                                                  \
  cudaError_t NAME(int cd, int cg, int sched, int tn, const LaunchPlan& lp) {           \
    if (cg == 1 && tn == 256) {                                                          \
      if (sched == SCHED_STATIC) B200_DISPATCH_CD(AB, 1, SCHED_STATIC, 256);             \
      if (sched == SCHED_CLC) B200_DISPATCH_CD(AB, 1, SCHED_CLC, 256);                   \
    } else if (cg == 2 && tn == 128) {                                                   \
      if (sched == SCHED_STATIC) B200_DISPATCH_CD(AB, 2, SCHED_STATIC, 128);             \
      if (sched == SCHED_CLC) B200_DISPATCH_CD(AB, 2, SCHED_CLC, 128);                   \
      if (sched == SCHED_STREAMK) B200_DISPATCH_CD(AB, 2, SCHED_STREAMK, 128);           \
    } else if (cg == 2 && tn == 256) {                                                   \
      if (sched == SCHED_STATIC) B200_DISPATCH_CD(AB, 2, SCHED_STATIC, 256);             \
      if (sched == SCHED_CLC) B200_DISPATCH_CD(AB, 2, SCHED_CLC, 256);                   \
      if (sched == SCHED_STREAMK) B200_DISPATCH_CD(AB, 2, SCHED_STREAMK, 256);           \
    } else if (cg == 2 && tn == 512) {                                                   \
      if (sched == SCHED_STATIC) B200_DISPATCH_CD(AB, 2, SCHED_STATIC, 512);             \
      if (sched == SCHED_CLC) B200_DISPATCH_CD(AB, 2, SCHED_CLC, 512);                   \
    }                                                                                    \
    return cudaErrorNotSupported;                                                        \
  }

}  // namespace b200
