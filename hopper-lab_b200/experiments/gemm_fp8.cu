// gemm_fp8 — B200 counterpart of the reference's 07_fp8 experiment
// (src/07_fp8/gemm_fp8.cu:225-300): e4m3 GEMM on tcgen05.mma kind::f8f6f4.
//
// CHECK: the reference's unscaled CHECK (512x512x256 e4m3, seeds 901/902, fp32 C,
//        3e-2/3e-2, x3) for every variant; BASELINE config 4 (2048^3, uniform seeds
//        903/904 quantised on the device with per-tensor scale = amax/448, bf16 C):
//        the device quantiser against the host one (bit-exact) and the GEMM against
//        the host GEMM on the dequantised inputs (3e-2, atol = 3e-2 * rms).
// GEMM : 2048^3 and 8192^3 scaled e4m3 -> bf16 over variants -> results/gemm_fp8_*.csv.
#include <algorithm>

#include "exp_common.h"

using namespace exp_common;

namespace {

// Host form of the per-tensor quantiser: scale = amax/448 (1 if all zero), q = e4m3(x/scale).
float host_quantize(const std::vector<float>& x, std::vector<__nv_fp8_e4m3>& q) {
  float amax = 0.f;
  for (float v : x) amax = std::max(amax, std::fabs(v));
  const float scale = amax > 0.f ? amax / 448.0f : 1.0f;
  q.resize(x.size());
  for (size_t i = 0; i < x.size(); ++i) q[i] = __nv_fp8_e4m3(x[i] / scale);
  return scale;
}

struct Scaled {
  int64_t M, N, K;
  void *dA = nullptr, *dB = nullptr;
  float *dsa = nullptr, *dsb = nullptr;
  std::vector<float> a_val, b_val;  // dequantised q values (without the scale)
  float sa = 1.f, sb = 1.f;
  bool quant_ok = true;
  Scaled(int64_t M_, int64_t N_, int64_t K_, uint32_t seed_a, uint32_t seed_b) : M(M_), N(N_), K(K_) {
    prep(hopper::make_random_vector(size_t(M * K), seed_a, -1.f, 1.f), &dA, &dsa, a_val, sa);
    prep(hopper::make_random_vector(size_t(N * K), seed_b, -1.f, 1.f), &dB, &dsb, b_val, sb);
  }
  ~Scaled() {
    cudaFree(dA);
    cudaFree(dB);
    cudaFree(dsa);
    cudaFree(dsb);
  }
  void prep(const std::vector<float>& x, void** dq, float** ds, std::vector<float>& val, float& s) {
    float* dx = nullptr;
    CUDA_CHECK(cudaMalloc(&dx, x.size() * 4));
    CUDA_CHECK(cudaMalloc(dq, x.size()));
    CUDA_CHECK(cudaMalloc(ds, 4));
    CUDA_CHECK(cudaMemcpy(dx, x.data(), x.size() * 4, cudaMemcpyHostToDevice));
    B200_CHECK(b200_quantize_e4m3(dx, int64_t(x.size()), *dq, *ds, nullptr));
    CUDA_CHECK(cudaDeviceSynchronize());
    cudaFree(dx);
    std::vector<__nv_fp8_e4m3> hq;
    s = host_quantize(x, hq);
    std::vector<__nv_fp8_e4m3> dqh(x.size());
    float dscale = 0.f;
    CUDA_CHECK(cudaMemcpy(dqh.data(), *dq, x.size(), cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(&dscale, *ds, 4, cudaMemcpyDeviceToHost));
    quant_ok = quant_ok && dscale == s && std::memcmp(dqh.data(), hq.data(), x.size()) == 0;
    val = to_float(hq);
  }
};

}  // namespace

int main(int argc, char** argv) {
  const Opts o = parse(argc, argv, "gemm_fp8: e4m3 tcgen05 GEMM with per-tensor scales (07_fp8)");
  auto caps = init_device();
  const double peak = peak_tflops(caps, B200_DT_E4M3);
  bool ok = true;
  {
    Problem p(B200_DT_E4M3, 512, 512, 256, 901, 902);
    auto ref = host_gemm(p.a_val, p.b_val, p.M, p.N, p.K);
    for (int v : {B200_VARIANT_1CTA, B200_VARIANT_PERSISTENT, B200_VARIANT_CLC, B200_VARIANT_2CTA,
                  B200_VARIANT_2CTA_CLC}) {
      char tag[64];
      std::snprintf(tag, sizeof(tag), "fp8 %s fp32 C x3", variant_name(v));
      ok = check(tag, p, B200_DT_F32, v, 0, 0, 0, ref, 3e-2, 3e-2) && ok;
    }
  }
  {
    Scaled p(2048, 2048, 2048, 903, 904);
    std::printf("[CHECK ] %-36s : %s\n", "device quantiser == host (bit-exact)", p.quant_ok ? "PASS" : "FAIL");
    ok = ok && p.quant_ok;
    auto ref = host_gemm(p.a_val, p.b_val, p.M, p.N, p.K);
    for (float& r : ref) r *= p.sa * p.sb;
    void* dC = nullptr;
    CUDA_CHECK(cudaMalloc(&dC, size_t(p.M * p.N) * 2));
    for (int v : {B200_VARIANT_PERSISTENT, B200_VARIANT_2CTA, B200_VARIANT_2CTA_CLC}) {
      auto a = args_for(B200_DT_E4M3, B200_DT_BF16, p.M, p.N, p.K, p.dA, p.dB, dC, v);
      a.scale_a = p.dsa;
      a.scale_b = p.dsb;
      run_checked(a);
      auto got = download_c(dC, B200_DT_BF16, size_t(p.M * p.N));
      auto rep = hopper::check_close(got, ref, 3e-2, 3e-2 * rms(ref));
      char tag[64];
      std::snprintf(tag, sizeof(tag), "config 4 scaled %s bf16 C", variant_name(v));
      hopper::print_report(rep, tag);
      ok = ok && rep.pass;
    }
    cudaFree(dC);
  }
  if (!ok) return 1;

  for (int64_t n : {int64_t(2048), int64_t(8192)}) {
    Scaled p(n, n, n, n == 2048 ? 903 : 905, n == 2048 ? 904 : 906);
    const double flops = 2.0 * double(n) * double(n) * double(n);
    std::printf("\n[GEMM  ] %lld^3 e4m3 -> bf16, per-tensor scales (peak %.0f TFLOPS)\n", (long long)n, peak);
    std::printf("  %-11s %-7s %12s %12s %10s %8s\n", "variant", "tile_n", "min_ms", "median_ms", "TFLOPS", "%peak");
    char path[64];
    std::snprintf(path, sizeof(path), "results/gemm_fp8_%lld.csv", (long long)n);
    hopper::CsvWriter csv(path, csv_columns());
    void* dC = nullptr;
    CUDA_CHECK(cudaMalloc(&dC, size_t(n * n) * 2));
    for (int v : {B200_VARIANT_1CTA, B200_VARIANT_PERSISTENT, B200_VARIANT_2CTA, B200_VARIANT_2CTA_CLC})
      for (int tn : {256, 512}) {
        if (tn == 512 && v != B200_VARIANT_2CTA && v != B200_VARIANT_2CTA_CLC) continue;
        if (o.quick && v == B200_VARIANT_1CTA) continue;
        auto a = args_for(B200_DT_E4M3, B200_DT_BF16, n, n, n, p.dA, p.dB, dC, v, 0, 0, tn);
        a.scale_a = p.dsa;
        a.scale_b = p.dsb;
        auto st = hopper::time_reps(3, n == 8192 ? 5 : 10, [&] { run(a); });
        const double tf = hopper::tflops(flops, st.min_ms);
        std::printf("  %-11s %-7d %12.3f %12.3f %10.2f %7.1f%%\n", variant_name(v), tn, st.min_ms, st.median_ms,
                    tf, 100.0 * tf / peak);
        csv_row(csv, v, tn, 0, 0, n, n, n, B200_DT_E4M3, 1, st, peak);
      }
    cudaFree(dC);
  }
  return 0;
}
