// errors.h — error-exit macros of the host harness (namespace-free macros, as in
// the reference's include/common/errors.h:8-19), plus B200_CHECK for the C ABI.
#pragma once

#include <cstdio>
#include <cstdlib>

#include <cuda_runtime.h>

#include "../b200gemm.h"

// Abort with file:line when a CUDA runtime call fails.
#define CUDA_CHECK(cmd)                                                                 \
  do {                                                                                  \
    const cudaError_t e__ = (cmd);                                                      \
    if (e__ != cudaSuccess) {                                                           \
      std::fprintf(stderr, "CUDA error %s:%d: %s (%s)\n", __FILE__, __LINE__,            \
                   cudaGetErrorString(e__), #cmd);                                      \
      std::exit(EXIT_FAILURE);                                                          \
    }                                                                                   \
  } while (0)

// Kernel launches report errors through cudaGetLastError().
#define CUDA_CHECK_LAST() CUDA_CHECK(cudaGetLastError())

// Abort with file:line when a b200gemm C-ABI call returns a negative code.
#define B200_CHECK(cmd)                                                                 \
  do {                                                                                  \
    const int rc__ = (cmd);                                                             \
    if (rc__ != B200_OK) {                                                              \
      std::fprintf(stderr, "b200gemm error %s:%d: %s (%d) (%s)\n", __FILE__, __LINE__,   \
                   b200_gemm_strerror(rc__), rc__, #cmd);                               \
      std::exit(EXIT_FAILURE);                                                          \
    }                                                                                   \
  } while (0)
