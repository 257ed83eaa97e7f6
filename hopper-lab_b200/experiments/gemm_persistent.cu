// gemm_persistent — B200 counterpart of the reference's 08_persistent experiments
// (src/08_persistent/gemm_fp8_persist.cu:272-360, gemm_fp8_bn128.cu:313-420):
// persistent tile schedules with group-M swizzle.
//
// The static schedule (grid = SMs, tile += grid) keeps the reference's tile_to_bmn
// order; the dynamic atomic tile queue becomes cluster-launch-control work
// stealing (clusterlaunchcontrol.try_cancel) in the CLC variants.
// CHECK: e4m3 512x512x256 and 2048x2048x256 (multi-wave), seeds 1001/1002, fp32 C,
//        3e-2, S x G matrix, x3 (gemm_fp8_persist.cu:282-318); seeds 2001/2002 for
//        the CLC variants (gemm_fp8_bn128.cu:323-351).
// GEMM : BASELINE config 5: e4m3 M = N = 8192, K in {1024, 4096, 16384} and skinny
//        M=256, N=16384, K=8192, bf16 C -> results/gemm_persistent.csv.
#include "exp_common.h"

using namespace exp_common;

int main(int argc, char** argv) {
  const Opts o = parse(argc, argv, "gemm_persistent: persistent / CLC tile schedulers (08_persistent)");
  auto caps = init_device();
  const double peak = peak_tflops(caps, B200_DT_E4M3);
  bool ok = true;
  for (int64_t n : {int64_t(512), int64_t(2048)}) {
    Problem p(B200_DT_E4M3, n, n, 256, 1001, 1002);
    auto ref = host_gemm(p.a_val, p.b_val, p.M, p.N, p.K);
    for (int v : {B200_VARIANT_PERSISTENT, B200_VARIANT_2CTA})
      for (int s = 2; s <= max_stages(v, B200_DT_E4M3); ++s)
        for (int g : {1, 8}) {
          char tag[64];
          std::snprintf(tag, sizeof(tag), "persist %lld %s S=%d G=%d", (long long)n, variant_name(v), s, g);
          ok = check(tag, p, B200_DT_F32, v, s, g, 0, ref, 3e-2, 3e-2) && ok;
        }
  }
  {
    Problem p(B200_DT_E4M3, 2048, 2048, 256, 2001, 2002);
    auto ref = host_gemm(p.a_val, p.b_val, p.M, p.N, p.K);
    for (int v : {B200_VARIANT_CLC, B200_VARIANT_2CTA_CLC})
      for (int g : {1, 8}) {
        char tag[64];
        std::snprintf(tag, sizeof(tag), "dynamic %s G=%d", variant_name(v), g);
        ok = check(tag, p, B200_DT_F32, v, 0, g, 0, ref, 3e-2, 3e-2) && ok;
      }
  }
  if (!ok) return 1;

  struct Shape { int64_t m, n, k; };
  const Shape shapes[] = {{8192, 8192, 1024}, {8192, 8192, 4096}, {8192, 8192, 16384}, {256, 16384, 8192}};
  hopper::CsvWriter csv("results/gemm_persistent.csv", csv_columns());
  std::printf("\n[GEMM  ] config 5: e4m3 -> bf16 (peak %.0f TFLOPS)\n", peak);
  std::printf("  %-20s %-11s %-7s %-5s %12s %12s %10s %8s\n", "shape", "variant", "tile_n", "G", "min_ms",
              "median_ms", "TFLOPS", "%peak");
  for (const Shape& sh : shapes) {
    Problem p(B200_DT_E4M3, sh.m, sh.n, sh.k, 1003, 1004);
    const double flops = 2.0 * double(sh.m) * double(sh.n) * double(sh.k);
    char shape[32];
    std::snprintf(shape, sizeof(shape), "%lldx%lldx%lld", (long long)sh.m, (long long)sh.n, (long long)sh.k);
    for (int v : {B200_VARIANT_PERSISTENT, B200_VARIANT_CLC, B200_VARIANT_2CTA, B200_VARIANT_2CTA_CLC})
      for (int tn : {256, 512})
        for (int g : {1, 8}) {
          if (tn == 512 && v != B200_VARIANT_2CTA && v != B200_VARIANT_2CTA_CLC) continue;
          if (o.quick && (g == 1 || tn == 512)) continue;
          auto st = time_case(p, B200_DT_BF16, v, 0, g, tn, 3, 5);
          const double tf = hopper::tflops(flops, st.min_ms);
          std::printf("  %-20s %-11s %-7d %-5d %12.3f %12.3f %10.2f %7.1f%%\n", shape, variant_name(v), tn, g,
                      st.min_ms, st.median_ms, tf, 100.0 * tf / peak);
          csv_row(csv, v, tn, 0, g, p, st, peak);
        }
  }
  return 0;
}
