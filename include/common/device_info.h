// device_info.h — device capability query of the host harness. Same names and
// fields as the reference's include/common/device_info.h:10-75 (DeviceCaps,
// query_device, theoretical_bw_gbps, print_device_caps, require_hopper); the
// clocks come from cudaDeviceGetAttribute because the cudaDeviceProp clock fields
// are deprecated. require_blackwell() is the check this build's executables use.
#pragma once

#include <cstdio>
#include <cstdlib>

#include <cuda_runtime.h>

#include "errors.h"

namespace hopper {

struct DeviceCaps {
  char name[256];
  int cc_major, cc_minor;
  int sm_count;
  int clock_khz;               // SM clock
  size_t total_mem;            // bytes
  size_t l2_bytes;
  int smem_per_block_default;  // KB
  int smem_per_block_optin;    // KB
  int smem_per_sm;             // KB
  int mem_clock_khz;
  int mem_bus_bits;
  int cluster_launch;
};

inline DeviceCaps query_device(int device_id = 0) {
  cudaDeviceProp p;
  CUDA_CHECK(cudaGetDeviceProperties(&p, device_id));
  DeviceCaps c{};
  std::snprintf(c.name, sizeof(c.name), "%s", p.name);
  c.cc_major = p.major;
  c.cc_minor = p.minor;
  c.sm_count = p.multiProcessorCount;
  CUDA_CHECK(cudaDeviceGetAttribute(&c.clock_khz, cudaDevAttrClockRate, device_id));
  CUDA_CHECK(cudaDeviceGetAttribute(&c.mem_clock_khz, cudaDevAttrMemoryClockRate, device_id));
  CUDA_CHECK(cudaDeviceGetAttribute(&c.mem_bus_bits, cudaDevAttrGlobalMemoryBusWidth, device_id));
  c.total_mem = p.totalGlobalMem;
  c.l2_bytes = size_t(p.l2CacheSize);
  c.smem_per_block_default = int(p.sharedMemPerBlock / 1024);
  c.smem_per_block_optin = int(p.sharedMemPerBlockOptin / 1024);
  c.smem_per_sm = int(p.sharedMemPerMultiprocessor / 1024);
  c.cluster_launch = p.clusterLaunch;
  return c;
}

// DDR estimate of the peak DRAM bandwidth, GB/s (for reference only).
inline double theoretical_bw_gbps(const DeviceCaps& c) {
  return 2.0 * double(c.mem_clock_khz) * 1e3 * (double(c.mem_bus_bits) / 8.0) / 1e9;
}

// Dense tensor peak in TFLOPS at the reported SM clock: SMs x clock x FLOP/clk/SM,
// with 8192 (f16/bf16) or 16384 (e4m3) dense FLOP per clock per SM on sm_100.
inline double dense_peak_tflops(const DeviceCaps& c, bool fp8) {
  const double per_sm = fp8 ? 16384.0 : 8192.0;
  return double(c.sm_count) * double(c.clock_khz) * 1e3 * per_sm / 1e12;
}

inline void print_device_caps(const DeviceCaps& c) {
  std::printf("=== Device ===\n");
  std::printf("  name                  : %s (cc %d.%d)\n", c.name, c.cc_major, c.cc_minor);
  std::printf("  SM count              : %d @ %.0f MHz\n", c.sm_count, c.clock_khz / 1000.0);
  std::printf("  global memory         : %.1f GB, L2 %zu KB\n",
              double(c.total_mem) / (1024.0 * 1024.0 * 1024.0), c.l2_bytes / 1024);
  std::printf("  shared mem / block    : %d KB (default) / %d KB (optin), per SM %d KB\n",
              c.smem_per_block_default, c.smem_per_block_optin, c.smem_per_sm);
  std::printf("  memory bus            : %d-bit @ %.2f GHz (~%.0f GB/s peak)\n", c.mem_bus_bits,
              c.mem_clock_khz / 1e6, theoretical_bw_gbps(c));
  std::printf("  cluster launch        : %s\n", c.cluster_launch ? "yes" : "no");
}

// Kept for source compatibility with the reference's experiments: passes on sm_90+.
inline void require_hopper(const DeviceCaps& c) {
  if (c.cc_major < 9) {
    std::fprintf(stderr, "needs sm_90 or newer; found %s (cc %d.%d)\n", c.name, c.cc_major,
                 c.cc_minor);
    std::exit(EXIT_FAILURE);
  }
}

// This build's kernels are compiled for sm_100a only.
inline void require_blackwell(const DeviceCaps& c) {
  if (c.cc_major != 10) {
    std::fprintf(stderr, "needs a Blackwell datacenter GPU (sm_100); found %s (cc %d.%d)\n", c.name,
                 c.cc_major, c.cc_minor);
    std::exit(EXIT_FAILURE);
  }
}

}  // namespace hopper
