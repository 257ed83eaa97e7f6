// gemm_internal.h — host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "b200gemm.h"
#include "gemm_sm100.cuh"

namespace b200 {

// Argument checks that need no GPU (same codes as b200_gemm).
int gemm_validate(const B200GemmArgs* a);

// Resolve the driver's tensor-map encoder once per process (allocates nothing).
int gemm_resolve_driver();

// Launch body shared by the entry points: `a` is validated with M, N > 0; `sms`
// and `cc_major` describe the current device; `status` is the device word the
// kernel's bounded waits report into.
// `allow_workspace` = false keeps the launch away from every schedule that needs
// library-owned device memory (stream-K): AUTO never picks it, an explicit request
// returns B200_ERR_SCRATCH_LIMIT.
// Fused all-gather of C (b200_gemm_allgather); validated by the caller.
struct GatherSpec {
  const void* dst;
  uint32_t mode;   // B200_GATHER_MULTICAST or B200_GATHER_PEERS
  uint32_t peers;  // pointers in the array (GATHER_PEERS)
  uint64_t ld;     // row pitch of the gathered matrix, elements
  uint64_t col;    // this GPU's first column, elements
};

int gemm_launch_impl(const B200GemmArgs& a, cudaStream_t stream, int sms, int cc_major,
                     uint32_t* status, bool allow_workspace = true, const GatherSpec* gather = nullptr);

// A launch with everything resolved: variant, tensor maps, kernel parameters, grid.
struct Prepared {
  alignas(64) CUtensorMap tA;
  alignas(64) CUtensorMap tB;
  alignas(64) CUtensorMap tC;
  KParams kp;
  uint32_t grid, smem;
  int ab, cd, cg, sched, tn;
  int dev;
  bool streamk;      // takes a fresh workspace epoch per launch
  bool memset_only;  // K == 0: C = 0
  void* c;
  size_t c_pitch, c_width, c_height;
};

int gemm_prepare(const B200GemmArgs& a, int sms, int cc_major, uint32_t* status, bool allow_workspace,
                 const GatherSpec* gather, Prepared* out);
int gemm_launch_prepared(Prepared& pr, cudaStream_t stream);

}  // namespace b200
