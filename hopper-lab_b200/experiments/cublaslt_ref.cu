// cublaslt_ref — the cuBLASLt reference column, B200 counterpart of the
// reference's 03_compute/cublas_gemm.cu:86-102 (cublasGemmEx column-major NN,
// fp16 in / fp16 out, compute 32F). Here: cuBLASLt on this build's TN layout (A
// M x K row-major, B N x K row-major, C M x N row-major) for fp16 -> fp16,
// bf16 -> bf16 and e4m3 -> bf16 with per-tensor scale pointers, at the BASELINE
// shapes, beside b200_gemm on the same buffers. cuBLASLt is a closed library and
// is only a reference column here, never on the b200gemm path.
//
// Row-major C = A . B^T is column-major C^T = B . A^T: cuBLASLt's "A" is our B with
// op T (K x N column-major, ld K), its "B" is our A with op N (K x M, ld K).
#include <cublasLt.h>

#include "exp_common.h"

using namespace exp_common;

#define LT_CHECK(x)                                                                        \
  do {                                                                                     \
    cublasStatus_t s__ = (x);                                                              \
    if (s__ != CUBLAS_STATUS_SUCCESS) {                                                    \
      std::fprintf(stderr, "cuBLASLt error %d at %s:%d (%s)\n", int(s__), __FILE__, __LINE__, #x); \
      std::exit(EXIT_FAILURE);                                                             \
    }                                                                                      \
  } while (0)

namespace {

struct LtGemm {
  cublasLtHandle_t h = nullptr;
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
  cublasLtMatmulHeuristicResult_t heur{};
  void* ws = nullptr;
  size_t ws_bytes = 64u << 20;
  LtGemm(int ab, int cd, int64_t M, int64_t N, int64_t K, const float* sa, const float* sb) {
    LT_CHECK(cublasLtCreate(&h));
    const cudaDataType_t tin = ab == B200_DT_F16 ? CUDA_R_16F : ab == B200_DT_BF16 ? CUDA_R_16BF : CUDA_R_8F_E4M3;
    const cudaDataType_t tout = cd == B200_DT_F16 ? CUDA_R_16F : CUDA_R_16BF;
    LT_CHECK(cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F));
    const cublasOperation_t tA = CUBLAS_OP_T, tB = CUBLAS_OP_N;
    LT_CHECK(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &tA, sizeof(tA)));
    LT_CHECK(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tB, sizeof(tB)));
    if (ab == B200_DT_E4M3) {
      // cuBLASLt's A is our B, its B is our A: swap the scale pointers accordingly
      LT_CHECK(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_A_SCALE_POINTER, &sb, sizeof(sb)));
      LT_CHECK(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_B_SCALE_POINTER, &sa, sizeof(sa)));
    }
    LT_CHECK(cublasLtMatrixLayoutCreate(&la, tin, uint64_t(K), uint64_t(N), K));
    LT_CHECK(cublasLtMatrixLayoutCreate(&lb, tin, uint64_t(K), uint64_t(M), K));
    LT_CHECK(cublasLtMatrixLayoutCreate(&lc, tout, uint64_t(N), uint64_t(M), N));
    CUDA_CHECK(cudaMalloc(&ws, ws_bytes));
    cublasLtMatmulPreference_t pref;
    LT_CHECK(cublasLtMatmulPreferenceCreate(&pref));
    LT_CHECK(cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws_bytes,
                                                  sizeof(ws_bytes)));
    int found = 0;
    LT_CHECK(cublasLtMatmulAlgoGetHeuristic(h, op, la, lb, lc, lc, pref, 1, &heur, &found));
    cublasLtMatmulPreferenceDestroy(pref);
    if (!found) {
      std::fprintf(stderr, "cuBLASLt: no algorithm\n");
      std::exit(EXIT_FAILURE);
    }
  }
  ~LtGemm() {
    cudaFree(ws);
    cublasLtMatrixLayoutDestroy(la);
    cublasLtMatrixLayoutDestroy(lb);
    cublasLtMatrixLayoutDestroy(lc);
    cublasLtMatmulDescDestroy(op);
    cublasLtDestroy(h);
  }
  void run(const void* A, const void* B, void* C) {
    const float one = 1.f, zero = 0.f;
    LT_CHECK(cublasLtMatmul(h, op, &one, B, la, A, lb, &zero, C, lc, C, lc, &heur.algo, ws, ws_bytes, nullptr));
  }
};

}  // namespace

int main(int argc, char** argv) {
  const Opts o = parse(argc, argv, "cublaslt_ref: cuBLASLt reference column beside b200_gemm (03_compute)");
  auto caps = init_device();
  hopper::CsvWriter csv("results/cublaslt_ref.csv",
                        {"impl", "dtype", "M", "N", "K", "min_ms", "median_ms", "tflops", "pct_peak", "peak_tflops"});
  struct Case { int ab, cd; int64_t m, n, k; };
  std::vector<Case> cases = {{B200_DT_F16, B200_DT_F16, 2048, 2048, 2048},
                             {B200_DT_F16, B200_DT_F16, 8192, 8192, 8192},
                             {B200_DT_BF16, B200_DT_BF16, 8192, 8192, 8192},
                             {B200_DT_E4M3, B200_DT_BF16, 2048, 2048, 2048},
                             {B200_DT_E4M3, B200_DT_BF16, 8192, 8192, 8192},
                             {B200_DT_E4M3, B200_DT_BF16, 8192, 8192, 1024},
                             {B200_DT_E4M3, B200_DT_BF16, 256, 16384, 8192}};
  if (o.quick) cases.resize(2);
  float *dsa = nullptr, *dsb = nullptr;
  CUDA_CHECK(cudaMalloc(&dsa, 4));
  CUDA_CHECK(cudaMalloc(&dsb, 4));
  const float half = 0.5f;
  CUDA_CHECK(cudaMemcpy(dsa, &half, 4, cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(dsb, &half, 4, cudaMemcpyHostToDevice));
  std::printf("\n[GEMM  ] cuBLASLt vs b200_gemm (TN, min over reps)\n");
  std::printf("  %-6s %-20s %12s %10s %12s %10s %9s\n", "dtype", "shape", "cublas_ms", "TFLOPS", "b200_ms", "TFLOPS",
              "b200/cub");
  bool ok = true;
  for (const Case& c : cases) {
    Problem p(c.ab, c.m, c.n, c.k, 605, 606);
    const double flops = 2.0 * double(c.m) * double(c.n) * double(c.k);
    const double peak = peak_tflops(caps, c.ab);
    void *dC = nullptr, *dR = nullptr;
    CUDA_CHECK(cudaMalloc(&dC, size_t(c.m * c.n) * 2));
    CUDA_CHECK(cudaMalloc(&dR, size_t(c.m * c.n) * 2));
    const float* sa = c.ab == B200_DT_E4M3 ? dsa : nullptr;
    const float* sb = c.ab == B200_DT_E4M3 ? dsb : nullptr;
    LtGemm lt(c.ab, c.cd, c.m, c.n, c.k, sa, sb);
    const int reps = c.m * c.n * c.k >= (int64_t(1) << 36) ? 10 : 30;
    auto st_c = hopper::time_reps(3, reps, [&] { lt.run(p.dA, p.dB, dR); });
    auto st_b = time_case(p, c.cd, B200_VARIANT_AUTO, 0, 0, 0, 3, reps, sa, sb);
    // both results on the same inputs: relative difference of the two outputs
    auto a = args_for(c.ab, c.cd, c.m, c.n, c.k, p.dA, p.dB, dC, B200_VARIANT_AUTO);
    a.scale_a = sa;
    a.scale_b = sb;
    run_checked(a);
    lt.run(p.dA, p.dB, dR);
    CUDA_CHECK(cudaDeviceSynchronize());
    auto x = download_c(dC, c.cd, size_t(c.m * c.n));
    auto y = download_c(dR, c.cd, size_t(c.m * c.n));
    const double rel = hopper::norm_rel_error(x, y);
    ok = ok && rel < (c.ab == B200_DT_E4M3 ? 3e-2 : 1e-2);
    const double tc = hopper::tflops(flops, st_c.min_ms), tb = hopper::tflops(flops, st_b.min_ms);
    char shape[32];
    std::snprintf(shape, sizeof(shape), "%lldx%lldx%lld", (long long)c.m, (long long)c.n, (long long)c.k);
    std::printf("  %-6s %-20s %12.3f %10.2f %12.3f %10.2f %8.3fx  (|b200-cublas|/|cublas| = %.1e)\n",
                dtype_name(c.ab), shape, st_c.min_ms, tc, st_b.min_ms, tb, tb / tc, rel);
    csv.row({"cublaslt", dtype_name(c.ab), std::to_string(c.m), std::to_string(c.n), std::to_string(c.k),
             std::to_string(st_c.min_ms), std::to_string(st_c.median_ms), std::to_string(tc),
             std::to_string(tc / peak), std::to_string(peak)});
    csv.row({"b200", dtype_name(c.ab), std::to_string(c.m), std::to_string(c.n), std::to_string(c.k),
             std::to_string(st_b.min_ms), std::to_string(st_b.median_ms), std::to_string(tb),
             std::to_string(tb / peak), std::to_string(peak)});
    cudaFree(dC);
    cudaFree(dR);
  }
  std::printf("[CHECK ] %-36s : %s\n", "b200_gemm agrees with cuBLASLt", ok ? "PASS" : "FAIL");
  cudaFree(dsa);
  cudaFree(dsb);
  return ok ? 0 : 1;
}
