// peak_tcgen05 — dense tensor-core peak microbenchmark, B200 counterpart of the
// reference's 03_compute/peak_flops.cu (mma.sync m16n8k16 f16 peak, :36-54).
//
// Every SM issues back-to-back tcgen05.mma on shared-memory operands that stay
// resident (no loads in the loop), M = 128 (1 CTA) or 256 (CTA pair), N = 256, into
// one TMEM accumulator; one commit at the end, a bounded wait, and clock64 around
// the loop. It reports dense FLOP per SM clock and TFLOPS, confirming the per-SM
// rates (f16/bf16 and e4m3) behind the "% of dense peak" figures of the GEMMs.
#include "exp_common.h"
#include "sm100_ptx.cuh"

using namespace exp_common;

namespace {

constexpr uint32_t kThreads = 128;

template <int KIND, int CG>
__global__ void __launch_bounds__(kThreads, 1)
    peak_kernel(uint32_t iters, unsigned long long* cycles, uint32_t* status, uint64_t wait_ns) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t abort_flag;
  const uint32_t raw = b200::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* basep = smem_raw + (base - raw);
  const uint32_t a_bytes = 128u * 128u, b_bytes = (256u / CG) * 128u;
  for (uint32_t i = threadIdx.x; i < (a_bytes + b_bytes) / 16u; i += blockDim.x)
    reinterpret_cast<uint4*>(basep)[i] = make_uint4(0x3c003c00u, 0x3c003c00u, 0x3c003c00u, 0x3c003c00u);
  const uint32_t rank = CG == 2 ? b200::cluster_ctarank() : 0u;
  const uint32_t bar_a = b200::smem_u32(&bar);
  if (threadIdx.x == 0) {
    b200::mbar_init(bar_a, 1);
    abort_flag = 0;
    b200::fence_mbar_init();
  }
  b200::fence_proxy_async_shared();
  if (threadIdx.x < 32) {
    b200::tmem_alloc<CG>(b200::smem_u32(&tmem_slot), 256);
    b200::tmem_relinquish<CG>();
  }
  b200::tc_fence_before();
  if constexpr (CG == 2) b200::cluster_sync(); else __syncthreads();
  b200::tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0 && rank == 0) {
    constexpr uint32_t idesc = b200::idesc_f32acc(0, 0, 128 * CG, 256);
    const unsigned long long t0 = clock64();
    for (uint32_t it = 0; it < iters; ++it) {
#pragma unroll
      for (uint32_t k = 0; k < 4; ++k)
        b200::umma<CG, KIND>(tmem, b200::sdesc_k_sw128(base + 32u * k),
                             b200::sdesc_k_sw128(base + a_bytes + 32u * k), idesc, (it | k) != 0u);
    }
    b200::umma_commit<CG>(bar_a);
    if (!b200::mbar_wait_bounded(bar_a, 0, wait_ns)) atomicOr(status, 1u);
    cycles[blockIdx.x / CG] = clock64() - t0;
  }
  b200::tc_fence_before();
  if constexpr (CG == 2) b200::cluster_sync(); else __syncthreads();
  if (threadIdx.x < 32) {
    b200::tc_fence_after();
    b200::tmem_dealloc<CG>(tmem, 256);
  }
}

template <int KIND, int CG>
void run_peak(const hopper::DeviceCaps& caps, hopper::CsvWriter& csv, uint32_t iters) {
  const uint32_t grid = uint32_t(caps.sm_count) / CG * CG;
  const size_t smem = 1024 + 128 * 128 + (256 / CG) * 128;
  auto kern = peak_kernel<KIND, CG>;
  CUDA_CHECK(cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  unsigned long long* dcyc = nullptr;
  uint32_t* dst = nullptr;
  CUDA_CHECK(cudaMalloc(&dcyc, sizeof(unsigned long long) * grid));
  CUDA_CHECK(cudaMalloc(&dst, 4));
  CUDA_CHECK(cudaMemset(dst, 0, 4));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  if (CG == 2) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  auto launch = [&] {
    CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, iters, dcyc, dst, uint64_t(2000000000ull)));
  };
  auto st = hopper::time_reps(2, 5, launch);
  uint32_t bad = 0;
  CUDA_CHECK(cudaMemcpy(&bad, dst, 4, cudaMemcpyDeviceToHost));
  std::vector<unsigned long long> cyc(grid / CG);
  CUDA_CHECK(cudaMemcpy(cyc.data(), dcyc, cyc.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
  double mean_cyc = 0;
  for (auto c : cyc) mean_cyc += double(c);
  mean_cyc /= double(cyc.size());
  const double kmma = KIND == 0 ? 16.0 : 32.0;
  const double flops_per_issuer = double(iters) * 4.0 * 2.0 * 128.0 * CG * 256.0 * kmma;
  const double per_sm_clk = flops_per_issuer / CG / mean_cyc;
  const double total = flops_per_issuer * double(grid / CG);
  const double tf = hopper::tflops(total, st.min_ms);
  const char* kind = KIND == 0 ? "f16/bf16" : "e4m3";
  char tag[64];
  std::snprintf(tag, sizeof(tag), "tcgen05 %s cta_group::%d", kind, CG);
  std::printf("[BENCH ] %-36s : %8.0f FLOP/clk/SM  %9.2f TFLOPS (min of 5)  %s\n", tag, per_sm_clk, tf,
              bad ? "WAIT TIMED OUT" : "");
  csv.row({kind, std::to_string(CG), std::to_string(iters), std::to_string(per_sm_clk), std::to_string(tf),
           std::to_string(st.min_ms), std::to_string(caps.sm_count), std::to_string(caps.clock_khz / 1000)});
  cudaFree(dcyc);
  cudaFree(dst);
  if (bad) std::exit(EXIT_FAILURE);
}

}  // namespace

int main(int argc, char** argv) {
  const Opts o = parse(argc, argv, "peak_tcgen05: dense tcgen05.mma peak per SM (03_compute)");
  auto caps = init_device();
  hopper::CsvWriter csv("results/peak_tcgen05.csv",
                        {"kind", "cta_group", "iters", "flop_per_clk_per_sm", "tflops", "min_ms", "sms", "max_mhz"});
  const uint32_t iters = o.quick ? 2000 : 20000;
  run_peak<0, 1>(caps, csv, iters);
  run_peak<0, 2>(caps, csv, iters);
  run_peak<1, 1>(caps, csv, iters);
  run_peak<1, 2>(caps, csv, iters);
  std::printf("  nominal dense: f16/bf16 8192 FLOP/clk/SM, e4m3 16384 -> %.0f / %.0f TFLOPS at %.0f MHz\n",
              hopper::dense_peak_tflops(caps, false), hopper::dense_peak_tflops(caps, true), caps.clock_khz / 1e3);
  return 0;
}
