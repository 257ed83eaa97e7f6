// tensor.h — seeded host inputs and an RAII device buffer. Same API as the
// reference's include/common/tensor.h:12-51 (make_random_vector, DeviceBuffer<T>);
// make_normal_vector adds the normal(mean, stddev) inputs of the bf16 config.
#pragma once

#include <cstdint>
#include <random>
#include <vector>

#include <cuda_runtime.h>

#include "errors.h"

namespace hopper {

// n floats from std::mt19937(seed) through std::uniform_real_distribution<float>(lo, hi).
inline std::vector<float> make_random_vector(size_t n, uint32_t seed = 0, float lo = -1.0f,
                                             float hi = 1.0f) {
  std::mt19937 gen(seed);
  std::uniform_real_distribution<float> u(lo, hi);
  std::vector<float> out(n);
  for (size_t i = 0; i < n; ++i) out[i] = u(gen);
  return out;
}

// n floats from std::mt19937(seed) through std::normal_distribution<float>(mean, stddev).
inline std::vector<float> make_normal_vector(size_t n, uint32_t seed, float mean, float stddev) {
  std::mt19937 gen(seed);
  std::normal_distribution<float> d(mean, stddev);
  std::vector<float> out(n);
  for (size_t i = 0; i < n; ++i) out[i] = d(gen);
  return out;
}

// Device allocation owned for the object's lifetime; not copyable.
template <typename T>
class DeviceBuffer {
 public:
  explicit DeviceBuffer(size_t n) : n_(n) {
    if (n_) CUDA_CHECK(cudaMalloc(&ptr_, n_ * sizeof(T)));
  }
  ~DeviceBuffer() {
    if (ptr_) cudaFree(ptr_);
  }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;

  void upload(const std::vector<T>& h) {
    CUDA_CHECK(cudaMemcpy(ptr_, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice));
  }
  std::vector<T> download() const {
    std::vector<T> h(n_);
    CUDA_CHECK(cudaMemcpy(h.data(), ptr_, n_ * sizeof(T), cudaMemcpyDeviceToHost));
    return h;
  }
  T* get() { return ptr_; }
  const T* get() const { return ptr_; }
  size_t size() const { return n_; }

 private:
  T* ptr_ = nullptr;
  size_t n_ = 0;
};

}  // namespace hopper
