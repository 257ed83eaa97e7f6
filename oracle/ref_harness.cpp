// ref_harness.cpp — builds oracle/_ref/libhopperref.so from the REFERENCE's own
// host headers. TEST INFRASTRUCTURE ONLY: used to pin the C restatement in
// gemm_oracle.c and to generate tests/golden fixtures.
//
// Compiled (oracle/Makefile, target `ref`) against
//   <reference>/include/common/tensor.h   make_random_vector (tensor.h:12-20)
//   <reference>/include/common/checker.h  check_close / CheckReport (checker.h:10-55)
// and the CUDA headers' host-side conversions that the reference's experiments use:
//   __half(float)          src/05_gemm/gemm_ws.cu:249
//   __nv_fp8_e4m3(float)   src/07_fp8/gemm_fp8.cu:182-186
//   __nv_bfloat16(float)   (bf16 config; the reference has no bf16 path)
// The GEMM loop itself sits inside the reference's main() functions of sm_90a
// .cu files (src/05_gemm/gemm_ws.cu:258-265), which cannot be compiled on their
// own; ref_gemm_loop below states the same three lines over the reference's
// own element types.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <cstdint>
#include <cstring>
#include <random>
#include <vector>

#include "common/checker.h"
#include "common/tensor.h"

extern "C" {

void ref_make_random_vector(uint32_t seed, int64_t n, float lo, float hi, float* out) {
  std::vector<float> v = hopper::make_random_vector(size_t(n), seed, lo, hi);
  std::memcpy(out, v.data(), sizeof(float) * size_t(n));
}

void ref_normal(uint32_t seed, int64_t n, float mean, float stddev, float* out) {
  std::mt19937 rng(seed);
  std::normal_distribution<float> dist(mean, stddev);
  for (int64_t i = 0; i < n; ++i) out[i] = dist(rng);
}

void ref_f32_to_f16(const float* x, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) {
    __half h(x[i]);
    std::memcpy(&out[i], &h, 2);
  }
}

void ref_f32_to_bf16(const float* x, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) {
    __nv_bfloat16 h(x[i]);
    std::memcpy(&out[i], &h, 2);
  }
}

void ref_f32_to_e4m3(const float* x, int64_t n, uint8_t* out) {
  for (int64_t i = 0; i < n; ++i) {
    __nv_fp8_e4m3 q(x[i]);
    std::memcpy(&out[i], &q, 1);
  }
}

void ref_e4m3_to_f32(const uint8_t* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    __nv_fp8_e4m3 q;
    std::memcpy(&q, &x[i], 1);
    out[i] = float(q);
  }
}

void ref_f16_to_f32(const uint16_t* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    __half h;
    std::memcpy(&h, &x[i], 2);
    out[i] = float(h);
  }
}

// The reference's host loop (src/05_gemm/gemm_ws.cu:258-265) over its fp16 inputs.
void ref_gemm_loop_f16(const uint16_t* a_bits, const uint16_t* b_bits, int64_t M, int64_t N, int64_t K,
                       float* ref) {
  const __half* a = reinterpret_cast<const __half*>(a_bits);
  const __half* b = reinterpret_cast<const __half*>(b_bits);
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.f;
      for (int64_t k = 0; k < K; ++k) acc += float(a[size_t(m) * K + k]) * float(b[size_t(n) * K + k]);
      ref[size_t(m) * N + n] = acc;
    }
}

// The same loop over e4m3 inputs (src/07_fp8/gemm_fp8.cu:246-253).
void ref_gemm_loop_e4m3(const uint8_t* a_bits, const uint8_t* b_bits, int64_t M, int64_t N, int64_t K,
                        float* ref) {
  const __nv_fp8_e4m3* a = reinterpret_cast<const __nv_fp8_e4m3*>(a_bits);
  const __nv_fp8_e4m3* b = reinterpret_cast<const __nv_fp8_e4m3*>(b_bits);
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.f;
      for (int64_t k = 0; k < K; ++k) acc += float(a[size_t(m) * K + k]) * float(b[size_t(n) * K + k]);
      ref[size_t(m) * N + n] = acc;
    }
}

// hopper::check_close on float vectors; returns pass and fills the report fields.
int ref_check_close(const float* got, const float* ref, int64_t n, double rtol, double atol,
                    int64_t* mismatches, double* max_abs, double* max_rel) {
  std::vector<float> g(got, got + n), e(ref, ref + n);
  hopper::CheckReport r = hopper::check_close(g, e, rtol, atol);
  *mismatches = int64_t(r.mismatches);
  *max_abs = r.max_abs_err;
  *max_rel = r.max_rel_err;
  return r.pass ? 1 : 0;
}

}  // extern "C"
