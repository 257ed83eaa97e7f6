// gemm_cluster — B200 counterpart of the reference's 06_cluster GEMMs
// (src/06_cluster/gemm_cluster.cu, gemm_ws_cluster.cu:50-218): the CTA pair.
//
// On Hopper the pair shared A through a TMA multicast (armed/empty_a protocol).
// Here the pair runs one cta_group::2 MMA (M = 256) and each CTA loads half of B;
// 256x512 pair tiles (tile_n = 512) share A between two N=256 MMAs as well.
// CHECK: 512x512x256 fp16 seeds 601/602 fp32 C (gemm_cluster.cu:196-229), and the
//        BASELINE config 3 (bf16 8192^3, normal(0,1)*0.1 seeds 605/606, bf16 C) on
//        seeded row bands, relative error <= 1e-2.
// GEMM : 2048^3 and 8192^3 bf16 over tile widths -> results/gemm_cluster_*.csv.
#include "exp_common.h"

using namespace exp_common;

int main(int argc, char** argv) {
  const Opts o = parse(argc, argv, "gemm_cluster: cta_group::2 pair GEMM (06_cluster)");
  auto caps = init_device();
  const double peak = peak_tflops(caps, B200_DT_BF16);
  bool ok = true;
  {
    Problem p(B200_DT_F16, 512, 512, 256, 601, 602);
    auto ref = host_gemm(p.a_val, p.b_val, p.M, p.N, p.K);
    for (int tn : {256, 512})
      for (int s = 2; s <= max_stages(B200_VARIANT_2CTA, B200_DT_F16, tn); ++s) {
        char tag[64];
        std::snprintf(tag, sizeof(tag), "pair %dw S=%d fp32 C x3", tn, s);
        ok = check(tag, p, B200_DT_F32, B200_VARIANT_2CTA, s, 0, tn, ref, 1e-3, 1e-3) && ok;
      }
  }
  {
    Problem p(B200_DT_BF16, 8192, 8192, 8192, 605, 606, /*normal=*/true);
    for (int64_t r0 : {int64_t(0), int64_t(4096), int64_t(8192 - 32)}) {
      auto ref = host_gemm(p.a_val, p.b_val, p.M, p.N, p.K, r0, r0 + 32);
      for (int tn : {256, 512}) {
        char tag[64];
        std::snprintf(tag, sizeof(tag), "config 3 rows %lld+32 %dw", (long long)r0, tn);
        ok = check(tag, p, B200_DT_BF16, B200_VARIANT_2CTA, 0, 0, tn, ref, 1e-2, 1e-2 * rms(ref), 1, r0,
                   32) && ok;
      }
    }
  }
  if (!ok) return 1;

  for (int64_t n : {int64_t(2048), int64_t(8192)}) {
    Problem p(B200_DT_BF16, n, n, n, 605, 606, true);
    const double flops = 2.0 * double(n) * double(n) * double(n);
    std::printf("\n[GEMM  ] %lld^3 bf16 -> bf16, CTA pair (peak %.0f TFLOPS)\n", (long long)n, peak);
    std::printf("  %-9s %-7s %-7s %12s %12s %10s %8s\n", "variant", "tile_n", "stages", "min_ms", "median_ms",
                "TFLOPS", "%peak");
    char path[64];
    std::snprintf(path, sizeof(path), "results/gemm_cluster_%lld.csv", (long long)n);
    hopper::CsvWriter csv(path, csv_columns());
    for (int v : {B200_VARIANT_2CTA, B200_VARIANT_2CTA_CLC})
      for (int tn : {256, 512})
        for (int g : {1, 8, 16}) {
          if (o.quick && g != 8) continue;
          auto st = time_case(p, B200_DT_BF16, v, 0, g, tn, 3, n == 8192 ? 5 : 10);
          const double tf = hopper::tflops(flops, st.min_ms);
          std::printf("  %-9s %-7d G=%-5d %12.3f %12.3f %10.2f %7.1f%%\n", variant_name(v), tn, g, st.min_ms,
                      st.median_ms, tf, 100.0 * tf / peak);
          csv_row(csv, v, tn, 0, g, p, st, peak);
        }
  }
  return 0;
}
