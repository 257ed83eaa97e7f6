// gemm_ws — B200 counterpart of the reference's 05_gemm experiment
// (src/05_gemm/gemm_ws.cu:239-353): the warp-specialised 1-CTA GEMM.
//
// CHECK: 512x512x256 fp16, seeds 601/602, fp32 C, rtol = atol = 1e-3, S in {2,3,4},
//        x3 reps (gemm_ws.cu:246-286); BASELINE config 1 (512^3 fp16 -> fp16 C) and
//        config 2 (2048^3 fp16 -> fp16 C), relative error <= 1e-2.
// GEMM : 2048x2048x1024 (seeds 603/604) and 8192^3 (seeds 605/606) over stages,
//        1-CTA and persistent tiles -> results/gemm_ws_{2048,8192}.csv.
#include "exp_common.h"

using namespace exp_common;

int main(int argc, char** argv) {
  const Opts o = parse(argc, argv, "gemm_ws: warp-specialised 1-CTA tcgen05 GEMM (05_gemm)");
  auto caps = init_device();
  const double peak = peak_tflops(caps, B200_DT_F16);
  bool ok = true;
  {
    Problem p(B200_DT_F16, 512, 512, 256, 601, 602);
    auto ref = host_gemm(p.a_val, p.b_val, p.M, p.N, p.K);
    for (int s : {2, 3, 4}) {
      char tag[64];
      std::snprintf(tag, sizeof(tag), "ws S=%d fp32 C x3", s);
      ok = check(tag, p, B200_DT_F32, B200_VARIANT_1CTA, s, 0, 0, ref, 1e-3, 1e-3) && ok;
    }
  }
  for (int64_t n : {int64_t(512), int64_t(2048)}) {
    Problem p(B200_DT_F16, n, n, n, n == 512 ? 601 : 603, n == 512 ? 602 : 604);
    auto ref = host_gemm(p.a_val, p.b_val, p.M, p.N, p.K);
    const double atol = 1e-2 * rms(ref);
    char tag[64];
    std::snprintf(tag, sizeof(tag), "config %d: %lld^3 fp16 C", n == 512 ? 1 : 2, (long long)n);
    ok = check(tag, p, B200_DT_F16, B200_VARIANT_1CTA, 0, 0, 0, ref, 1e-2, atol, 1) && ok;
  }
  if (!ok) return 1;

  struct Shape { int64_t m, n, k; uint32_t sa, sb; const char* csv; };
  const Shape shapes[] = {{2048, 2048, 1024, 603, 604, "results/gemm_ws_2048.csv"},
                          {8192, 8192, 8192, 605, 606, "results/gemm_ws_8192.csv"}};
  for (const Shape& sh : shapes) {
    Problem p(B200_DT_F16, sh.m, sh.n, sh.k, sh.sa, sh.sb);
    const double flops = 2.0 * double(sh.m) * double(sh.n) * double(sh.k);
    std::printf("\n[GEMM  ] %lldx%lldx%lld fp16 -> fp16 (peak %.0f TFLOPS at %.0f MHz)\n",
                (long long)sh.m, (long long)sh.n, (long long)sh.k, peak, caps.clock_khz / 1e3);
    std::printf("  %-11s %-7s %12s %12s %10s %8s\n", "variant", "stages", "min_ms", "median_ms", "TFLOPS",
                "%peak");
    hopper::CsvWriter csv(sh.csv, csv_columns());
    for (int v : {B200_VARIANT_1CTA, B200_VARIANT_PERSISTENT}) {
      for (int s = 2; s <= max_stages(v, B200_DT_F16); ++s) {
        if (o.quick && s != max_stages(v, B200_DT_F16)) continue;
        auto st = time_case(p, B200_DT_F16, v, s, 0, 0, 3, sh.m == 8192 ? 5 : 10);
        const double tf = hopper::tflops(flops, st.min_ms);
        std::printf("  %-11s %-7d %12.3f %12.3f %10.2f %7.1f%%\n", variant_name(v), s, st.min_ms,
                    st.median_ms, tf, 100.0 * tf / peak);
        csv_row(csv, v, 0, s, 0, p, st, peak);
      }
    }
  }
  return 0;
}
