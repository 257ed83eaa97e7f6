// quant.cu — on-GPU per-tensor e4m3 quantiser: amax reduction, scale = amax/448,
// q = e4m3_rn_satfinite(x / scale).
//
// The reference quantises on the host, without a scale, one element at a time
// (`quantize`, src/07_fp8/gemm_fp8.cu:182-186: q[i] = __nv_fp8_e4m3(f[i])). The
// build's fp8 configs add the per-tensor scale amax/448; this file is the device
// form of that step, the producer of the fp8 GEMM's A/B and scale pointers.
//
// Three launches, all HBM-bound streaming passes (9 bytes moved per element):
//   1. amax_kernel   : |x| max per block, atomicMax on the bit pattern into *scale
//                      (non-negative floats order like their bit patterns)
//   2. quant_kernel  : reads the amax from *scale, writes q
//   3. scale_kernel  : turns *scale from amax into amax/448 (1 when amax == 0)
#include <cuda_runtime.h>

#include <cstdint>

#include "b200gemm.h"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__global__ void __launch_bounds__(kThreads) amax_kernel(const float* __restrict__ x, int64_t n,
                                                        unsigned* __restrict__ amax_bits) {
  float m = 0.0f;
  const int64_t tid = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  const int64_t n4 = n / 4;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  for (int64_t i = tid; i < n4; i += stride) {
    const float4 v = __ldcs(x4 + i);
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  for (int64_t i = n4 * 4 + tid; i < n; i += stride) m = fmaxf(m, fabsf(x[i]));
  m = warp_max(m);
  __shared__ float red[kThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kThreads / 32 ? red[threadIdx.x] : 0.0f;
    v = warp_max(v);
    if (threadIdx.x == 0) atomicMax(amax_bits, __float_as_uint(v));
  }
}

__device__ __forceinline__ float scale_from_amax(float amax) {
  return amax > 0.0f ? amax / 448.0f : 1.0f;
}

// Two fp32 -> two e4m3 (RN, saturate to ±448), packed little-endian: lo in byte 0.
__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__global__ void __launch_bounds__(kThreads) quant_kernel(const float* __restrict__ x, int64_t n,
                                                         const unsigned* __restrict__ amax_bits,
                                                         uint8_t* __restrict__ q) {
  const float scale = scale_from_amax(__uint_as_float(*amax_bits));
  const int64_t tid = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  const int64_t n8 = n / 8;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  uint2* q8 = reinterpret_cast<uint2*>(q);
  for (int64_t i = tid; i < n8; i += stride) {
    const float4 a = __ldcs(x4 + 2 * i);
    const float4 b = __ldcs(x4 + 2 * i + 1);
    const uint32_t w0 = uint32_t(cvt_e4m3x2(a.x / scale, a.y / scale)) |
                        (uint32_t(cvt_e4m3x2(a.z / scale, a.w / scale)) << 16);
    const uint32_t w1 = uint32_t(cvt_e4m3x2(b.x / scale, b.y / scale)) |
                        (uint32_t(cvt_e4m3x2(b.z / scale, b.w / scale)) << 16);
    __stcs(q8 + i, make_uint2(w0, w1));
  }
  for (int64_t i = n8 * 8 + tid; i < n; i += stride) {
    q[i] = uint8_t(cvt_e4m3x2(x[i] / scale, 0.0f) & 0xFFu);
  }
}

__global__ void scale_kernel(float* scale) {
  const float amax = *scale;
  *scale = scale_from_amax(amax);
}

}  // namespace

extern "C" int b200_quantize_e4m3(const float* x, int64_t n, void* q, float* scale, void* stream_v) {
  if (n < 0) return B200_ERR_SHAPE;
  if (!scale || (n > 0 && (!x || !q))) return B200_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(q) & 7u) ||
      (reinterpret_cast<uintptr_t>(scale) & 3u))
    return B200_ERR_ALIGN;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return B200_ERR_CUDA;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return B200_ERR_CUDA;
  if (cudaMemsetAsync(scale, 0, sizeof(float), stream) != cudaSuccess) return B200_ERR_CUDA;
  if (n > 0) {
    // 8 resident 256-thread blocks per SM cover the grid-stride loops.
    const int64_t want = (n / 8 + kThreads - 1) / kThreads;
    const int64_t cap = int64_t(sms) * 8;
    const unsigned grid = unsigned(want < 1 ? 1 : (want < cap ? want : cap));
    unsigned* bits = reinterpret_cast<unsigned*>(scale);
    amax_kernel<<<grid, kThreads, 0, stream>>>(x, n, bits);
    quant_kernel<<<grid, kThreads, 0, stream>>>(x, n, bits, static_cast<uint8_t*>(q));
  }
  scale_kernel<<<1, 1, 0, stream>>>(scale);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_LAUNCH;
}
