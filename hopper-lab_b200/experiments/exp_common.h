// exp_common.h — shared pieces of the per-experiment executables.
//
// Each executable mirrors one of the reference's experiment mains
// (src/05_gemm/gemm_ws.cu:239-353, src/06_cluster/gemm_ws_cluster.cu,
// src/07_fp8/gemm_fp8.cu, src/08_persistent/gemm_fp8_persist.cu, …): query the
// device, build seeded host inputs with the harness, run the kernel through the
// C ABI, compare against a host GEMM with check_close and print [CHECK ] lines,
// time with time_reps and print a [GEMM  ] table, and append results/*.csv.
// The host GEMM below is the CHECK loop the reference's mains carry inline
// (acc += float(a[m*K+k]) * float(b[n*K+k]), fp32, sequential in k), spread
// over host threads by rows.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cmath>
#include <cstring>
#include <filesystem>
#include <string>
#include <thread>
#include <vector>

#include "b200gemm.h"
#include "common/bench.h"
#include "common/checker.h"
#include "common/device_info.h"
#include "common/errors.h"
#include "common/tensor.h"
#include "common/timer.h"

namespace exp_common {

struct Opts {
  bool quick = false;  // smaller timing set (CI / smoke runs)
};

inline Opts parse(int argc, char** argv, const char* what) {
  Opts o;
  for (int i = 1; i < argc; ++i) {
    if (!std::strcmp(argv[i], "--quick")) o.quick = true;
    if (!std::strcmp(argv[i], "--help") || !std::strcmp(argv[i], "-h")) {
      std::printf("%s\nusage: %s [--quick]\n", what, argv[0]);
      std::exit(0);
    }
  }
  return o;
}

inline hopper::DeviceCaps init_device() {
  auto caps = hopper::query_device();
  hopper::print_device_caps(caps);
  hopper::require_blackwell(caps);
  std::filesystem::create_directories("results");
  return caps;
}

// Element conversions of the reference's mains (CUDA headers' host conversions).
inline std::vector<__half> to_f16(const std::vector<float>& v) { return {v.begin(), v.end()}; }
inline std::vector<__nv_bfloat16> to_bf16(const std::vector<float>& v) {
  std::vector<__nv_bfloat16> r(v.size());
  for (size_t i = 0; i < v.size(); ++i) r[i] = __nv_bfloat16(v[i]);
  return r;
}
inline std::vector<__nv_fp8_e4m3> to_e4m3(const std::vector<float>& v) {
  std::vector<__nv_fp8_e4m3> r(v.size());
  for (size_t i = 0; i < v.size(); ++i) r[i] = __nv_fp8_e4m3(v[i]);
  return r;
}
template <typename T>
std::vector<float> to_float(const std::vector<T>& v) {
  std::vector<float> r(v.size());
  for (size_t i = 0; i < v.size(); ++i) r[i] = float(v[i]);
  return r;
}

// Host CHECK GEMM: rows [r0, r1) of C = A . B^T over fp32 values of the inputs.
inline std::vector<float> host_gemm(const std::vector<float>& a, const std::vector<float>& b, int64_t M,
                                    int64_t N, int64_t K, int64_t r0 = 0, int64_t r1 = -1) {
  if (r1 < 0) r1 = M;
  std::vector<float> c(size_t((r1 - r0) * N));
  const unsigned nt = std::max(1u, std::thread::hardware_concurrency());
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; ++t) {
    th.emplace_back([&, t] {
      for (int64_t m = r0 + t; m < r1; m += nt)
        for (int64_t n = 0; n < N; ++n) {
          float acc = 0.f;
          for (int64_t k = 0; k < K; ++k) acc += a[size_t(m * K + k)] * b[size_t(n * K + k)];
          c[size_t((m - r0) * N + n)] = acc;
        }
    });
  }
  for (auto& x : th) x.join();
  return c;
}

inline B200GemmArgs args_for(int ab, int cd, int64_t M, int64_t N, int64_t K, const void* A,
                             const void* B, void* C, int variant, int stages = 0, int group_m = 0,
                             int tile_n = 0) {
  B200GemmArgs a;
  std::memset(&a, 0, sizeof(a));
  a.ab_dtype = ab;
  a.c_dtype = cd;
  a.M = M;
  a.N = N;
  a.K = K;
  a.lda = K;
  a.ldb = K;
  a.ldc = N;
  a.A = A;
  a.B = B;
  a.C = C;
  a.variant = variant;
  a.stages = stages;
  a.group_m = group_m;
  a.tile_n = tile_n;
  return a;
}

inline void run(const B200GemmArgs& a) { B200_CHECK(b200_gemm(&a, nullptr)); }

// Launch + device status check (bounded waits must not have fired).
inline void run_checked(const B200GemmArgs& a) {
  run(a);
  uint32_t bits = 0;
  const int st = b200_gemm_status(nullptr, 1, &bits);
  if (st != B200_OK) {
    std::fprintf(stderr, "device status %s (bits 0x%x)\n", b200_gemm_strerror(st), bits);
    std::exit(EXIT_FAILURE);
  }
}

inline const char* variant_name(int v) {
  switch (v) {
    case B200_VARIANT_1CTA: return "1cta";
    case B200_VARIANT_2CTA: return "2cta";
    case B200_VARIANT_PERSISTENT: return "persistent";
    case B200_VARIANT_CLC: return "clc";
    case B200_VARIANT_2CTA_CLC: return "2cta_clc";
    case B200_VARIANT_2CTA_STREAMK: return "2cta_streamk";
    default: return "auto";
  }
}

inline int max_stages(int variant, int ab, int tile_n = 0) {
  int32_t tm, tn = tile_n, ms, ds;
  B200_CHECK(b200_gemm_variant_info(variant, ab, &tm, &tn, &ms, &ds));
  return ms;
}

// The BENCH line format of the reference's examples ([BENCH ] tag, checker.h style).
inline void print_bench(const char* tag, double ms, double flops) {
  std::printf("[BENCH ] %-36s : %10.3f ms  %10.2f TFLOPS\n", tag, ms, hopper::tflops(flops, ms));
}

}  // namespace exp_common

namespace exp_common {

// Device copies of a seeded problem in the element type `ab` (f16 / bf16 / e4m3,
// unscaled) plus the fp32 values the host CHECK GEMM uses.
struct Problem {
  int64_t M = 0, N = 0, K = 0;
  int ab = B200_DT_F16;
  std::vector<float> a_val, b_val;  // fp32 values of the narrow inputs
  void* dA = nullptr;
  void* dB = nullptr;
  Problem(const Problem&) = delete;
  Problem& operator=(const Problem&) = delete;
  Problem(int ab_, int64_t M_, int64_t N_, int64_t K_, uint32_t seed_a, uint32_t seed_b,
          bool normal = false)
      : M(M_), N(N_), K(K_), ab(ab_) {
    auto fa = normal ? hopper::make_normal_vector(size_t(M * K), seed_a, 0.f, 0.1f)
                     : hopper::make_random_vector(size_t(M * K), seed_a, -1.f, 1.f);
    auto fb = normal ? hopper::make_normal_vector(size_t(N * K), seed_b, 0.f, 0.1f)
                     : hopper::make_random_vector(size_t(N * K), seed_b, -1.f, 1.f);
    upload(fa, &dA, a_val);
    upload(fb, &dB, b_val);
  }
  ~Problem() {
    cudaFree(dA);
    cudaFree(dB);
  }

 private:
  void upload(const std::vector<float>& f, void** d, std::vector<float>& val) {
    size_t bytes = 0;
    if (ab == B200_DT_F16) {
      auto v = to_f16(f);
      val = to_float(v);
      bytes = v.size() * 2;
      CUDA_CHECK(cudaMalloc(d, bytes));
      CUDA_CHECK(cudaMemcpy(*d, v.data(), bytes, cudaMemcpyHostToDevice));
    } else if (ab == B200_DT_BF16) {
      auto v = to_bf16(f);
      val = to_float(v);
      bytes = v.size() * 2;
      CUDA_CHECK(cudaMalloc(d, bytes));
      CUDA_CHECK(cudaMemcpy(*d, v.data(), bytes, cudaMemcpyHostToDevice));
    } else {
      auto v = to_e4m3(f);
      val = to_float(v);
      bytes = v.size();
      CUDA_CHECK(cudaMalloc(d, bytes));
      CUDA_CHECK(cudaMemcpy(*d, v.data(), bytes, cudaMemcpyHostToDevice));
    }
  }
};

inline int c_bytes(int cd) { return cd == B200_DT_F32 ? 4 : 2; }

// Download C (any output type) as fp32.
inline std::vector<float> download_c(const void* dC, int cd, size_t n) {
  std::vector<float> out(n);
  if (cd == B200_DT_F32) {
    CUDA_CHECK(cudaMemcpy(out.data(), dC, n * 4, cudaMemcpyDeviceToHost));
  } else if (cd == B200_DT_F16) {
    std::vector<__half> h(n);
    CUDA_CHECK(cudaMemcpy(h.data(), dC, n * 2, cudaMemcpyDeviceToHost));
    out = to_float(h);
  } else {
    std::vector<__nv_bfloat16> h(n);
    CUDA_CHECK(cudaMemcpy(h.data(), dC, n * 2, cudaMemcpyDeviceToHost));
    out = to_float(h);
  }
  return out;
}

// One CHECK line: `reps` runs of the configuration against `ref` (rows [r0, r0+rows)).
inline bool check(const char* tag, const Problem& p, int cd, int variant, int stages, int group_m,
                  int tile_n, const std::vector<float>& ref, double rtol, double atol, int reps = 3,
                  int64_t r0 = 0, int64_t rows = -1) {
  if (rows < 0) rows = p.M;
  void* dC = nullptr;
  const size_t n = size_t(p.M * p.N);
  CUDA_CHECK(cudaMalloc(&dC, n * size_t(c_bytes(cd))));
  bool ok = true;
  for (int r = 0; r < reps; ++r) {
    CUDA_CHECK(cudaMemset(dC, 0xFF, n * size_t(c_bytes(cd))));  // NaN-filled
    run_checked(args_for(p.ab, cd, p.M, p.N, p.K, p.dA, p.dB, dC, variant, stages, group_m, tile_n));
    auto all = download_c(dC, cd, n);
    std::vector<float> got(all.begin() + r0 * p.N, all.begin() + (r0 + rows) * p.N);
    auto rep = hopper::check_close(got, ref, rtol, atol);
    for (float x : got)
      if (!(x == x)) {  // NaN: the check counts it as a failure
        rep.pass = false;
        ++rep.mismatches;
      }
    if (!rep.pass) {
      char t[96];
      std::snprintf(t, sizeof(t), "%s rep=%d", tag, r);
      hopper::print_report(rep, t);
    }
    ok = ok && rep.pass;
  }
  std::printf("[CHECK ] %-36s : %s\n", tag, ok ? "PASS" : "FAIL");
  cudaFree(dC);
  return ok;
}

// rtol = atol-relative check used for the 1e-2 configs: atol = tol * rms(ref).
inline double rms(const std::vector<float>& v) {
  double s = 0;
  for (float x : v) s += double(x) * double(x);
  return v.empty() ? 0.0 : std::sqrt(s / double(v.size()));
}

// Time one configuration: min and median over `reps` launches after `warmup`.
inline hopper::TimingStats time_case(const Problem& p, int cd, int variant, int stages, int group_m,
                                     int tile_n, int warmup, int reps, const float* sa = nullptr,
                                     const float* sb = nullptr) {
  void* dC = nullptr;
  CUDA_CHECK(cudaMalloc(&dC, size_t(p.M * p.N) * size_t(c_bytes(cd))));
  auto a = args_for(p.ab, cd, p.M, p.N, p.K, p.dA, p.dB, dC, variant, stages, group_m, tile_n);
  a.scale_a = sa;
  a.scale_b = sb;
  auto st = hopper::time_reps(warmup, reps, [&] { run(a); });
  uint32_t bits = 0;
  if (b200_gemm_status(nullptr, 1, &bits) != B200_OK) {
    std::fprintf(stderr, "device status bits 0x%x\n", bits);
    std::exit(EXIT_FAILURE);
  }
  cudaFree(dC);
  return st;
}

inline const char* dtype_name(int dt) {
  switch (dt) {
    case B200_DT_F16: return "f16";
    case B200_DT_BF16: return "bf16";
    case B200_DT_E4M3: return "e4m3";
    default: return "f32";
  }
}

// Row of the CSV schema every experiment writes (the reference's columns plus
// gpus, dtype, pct_peak and peak_tflops).
inline std::vector<std::string> csv_columns() {
  return {"variant", "tile_n", "stages", "group_m", "M", "N", "K", "dtype", "gpus", "min_ms", "median_ms",
          "tflops", "pct_peak", "peak_tflops"};
}

inline void csv_row(hopper::CsvWriter& w, int variant, int tile_n, int stages, int group_m, int64_t M,
                    int64_t N, int64_t K, int ab, int gpus, const hopper::TimingStats& st, double peak) {
  const double tf = hopper::tflops(2.0 * double(M) * double(N) * double(K), st.min_ms);
  w.row({variant_name(variant), std::to_string(tile_n ? tile_n : 256), std::to_string(stages),
         std::to_string(group_m), std::to_string(M), std::to_string(N), std::to_string(K), dtype_name(ab),
         std::to_string(gpus), std::to_string(st.min_ms), std::to_string(st.median_ms), std::to_string(tf),
         std::to_string(tf / peak), std::to_string(peak)});
}

inline void csv_row(hopper::CsvWriter& w, int variant, int tile_n, int stages, int group_m, const Problem& p,
                    const hopper::TimingStats& st, double peak) {
  csv_row(w, variant, tile_n, stages, group_m, p.M, p.N, p.K, p.ab, 1, st, peak);
}

// Dense tensor peak used for % of peak: SMs x max SM clock x dense FLOP/clk/SM.
inline double peak_tflops(const hopper::DeviceCaps& c, int ab) {
  return hopper::dense_peak_tflops(c, ab == B200_DT_E4M3);
}

}  // namespace exp_common
