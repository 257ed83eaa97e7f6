// timer.h — CUDA-event timing of the host harness. Same API as the reference's
// include/common/timer.h:17-73 (TimingStats, GpuTimer, time_reps) with an optional
// stream and a median in the statistics.
#pragma once

#include <algorithm>
#include <functional>
#include <vector>

#include <cuda_runtime.h>

#include "errors.h"

namespace hopper {

struct TimingStats {
  int reps = 0;
  double min_ms = 0.0;
  double mean_ms = 0.0;
  double max_ms = 0.0;
  double median_ms = 0.0;
};

class GpuTimer {
 public:
  explicit GpuTimer(cudaStream_t s = nullptr) : stream_(s) {
    CUDA_CHECK(cudaEventCreate(&a_));
    CUDA_CHECK(cudaEventCreate(&b_));
  }
  ~GpuTimer() {
    cudaEventDestroy(a_);
    cudaEventDestroy(b_);
  }
  GpuTimer(const GpuTimer&) = delete;
  GpuTimer& operator=(const GpuTimer&) = delete;

  void start() { CUDA_CHECK(cudaEventRecord(a_, stream_)); }
  void stop() { CUDA_CHECK(cudaEventRecord(b_, stream_)); }
  // Milliseconds between start() and stop(); waits for stop().
  double elapsed_ms() {
    CUDA_CHECK(cudaEventSynchronize(b_));
    float ms = 0.f;
    CUDA_CHECK(cudaEventElapsedTime(&ms, a_, b_));
    return double(ms);
  }

 private:
  cudaStream_t stream_;
  cudaEvent_t a_ = nullptr, b_ = nullptr;
};

// `warmup` untimed calls, then `reps` calls each timed on its own event pair.
inline TimingStats time_reps(int warmup, int reps, const std::function<void()>& launch,
                             cudaStream_t stream = nullptr) {
  for (int i = 0; i < warmup; ++i) launch();
  CUDA_CHECK(cudaDeviceSynchronize());
  std::vector<double> t(size_t(reps > 0 ? reps : 0));
  GpuTimer timer(stream);
  for (int i = 0; i < reps; ++i) {
    timer.start();
    launch();
    timer.stop();
    t[size_t(i)] = timer.elapsed_ms();
  }
  TimingStats s;
  s.reps = reps;
  if (reps <= 0) return s;
  double sum = 0.0;
  for (double x : t) sum += x;
  s.mean_ms = sum / reps;
  s.min_ms = *std::min_element(t.begin(), t.end());
  s.max_ms = *std::max_element(t.begin(), t.end());
  std::vector<double> u = t;
  std::sort(u.begin(), u.end());
  s.median_ms = (reps % 2) ? u[size_t(reps / 2)] : 0.5 * (u[size_t(reps / 2 - 1)] + u[size_t(reps / 2)]);
  return s;
}

}  // namespace hopper
