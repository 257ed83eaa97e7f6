// gemm_multi_gpu — BASELINE config 5's multi-GPU row: one GEMM with N split
// column-wise over the GPUs of one box (the reference has no multi-GPU code).
//
// One host thread per GPU. GPU g holds all of A (M x K, replicated), its contiguous
// row slab B[n0:n1, :] and writes its own C slab (M x (n1-n0)); the compute needs
// no exchange. Box TFLOPS = total flops / max over GPUs of the per-GPU kernel time
// (all GPUs start after a host barrier; CUDA events on each GPU's stream). An NCCL
// all-gather of the C slabs ([G][M][N/G]) and a re-layout kernel to row-major M x N
// are timed separately (--allgather).
// CHECK: a small fp16 problem (512 x 512*G x 1024, seeds 601/602) split the same
//        way, gathered and compared with the host GEMM (relative error <= 1e-2).
// GEMM : e4m3 M=16384, N=65536, K=8192, per-tensor scales, bf16 C; --gpus G
//        (default: all visible) -> results/gemm_multi_gpu.csv.
#include <nccl.h>

#include <barrier>
#include <mutex>

#include "exp_common.h"

using namespace exp_common;

#define NCCL_CHECK(x)                                                                     \
  do {                                                                                    \
    ncclResult_t r__ = (x);                                                               \
    if (r__ != ncclSuccess) {                                                             \
      std::fprintf(stderr, "NCCL error %s at %s:%d\n", ncclGetErrorString(r__), __FILE__, __LINE__); \
      std::exit(EXIT_FAILURE);                                                            \
    }                                                                                     \
  } while (0)

namespace {

// uniform[-1, 1) from a counter hash (splitmix64), for device-side inputs too large
// to generate on the host.
__global__ void fill_uniform(float* x, int64_t n, uint64_t seed) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    uint64_t z = seed + uint64_t(i) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    x[i] = float(int64_t(z >> 40) - (int64_t(1) << 23)) * (1.0f / float(1 << 23));
  }
}

// [G][M][Ng] (all-gathered slabs) -> row-major M x (G*Ng), 16-byte vectors.
__global__ void relayout(const uint4* src, uint4* dst, int64_t G, int64_t M, int64_t ng_vec) {
  const int64_t total = G * M * ng_vec;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t g = i / (M * ng_vec), rem = i % (M * ng_vec), m = rem / ng_vec, v = rem % ng_vec;
    dst[m * (G * ng_vec) + g * ng_vec + v] = src[i];
  }
}

struct Shard {
  int dev = 0;
  int64_t n0 = 0, n1 = 0;
  void *dA = nullptr, *dB = nullptr, *dC = nullptr;
  float *sa = nullptr, *sb = nullptr;
  cudaStream_t s = nullptr;
  double ms = 0.0;
};

std::pair<int64_t, int64_t> shard_columns(int64_t n, int world, int rank) {
  const int64_t units = (n + 15) / 16, base = units / world, extra = units % world;
  const int64_t u0 = rank * base + std::min<int64_t>(rank, extra);
  const int64_t u1 = u0 + base + (rank < extra ? 1 : 0);
  return {std::min(n, u0 * 16), std::min(n, u1 * 16)};
}

}  // namespace

int main(int argc, char** argv) {
  int gpus = 0;
  bool allgather = false;
  int64_t M = 16384, N = 65536, K = 8192;
  for (int i = 1; i < argc; ++i) {
    if (!std::strcmp(argv[i], "--gpus") && i + 1 < argc) gpus = std::atoi(argv[++i]);
    if (!std::strcmp(argv[i], "--allgather")) allgather = true;
    if (!std::strcmp(argv[i], "--quick")) { M = 4096; N = 16384; K = 4096; }
    if (!std::strcmp(argv[i], "--help")) {
      std::printf("gemm_multi_gpu: N-sharded e4m3 GEMM across GPUs\nusage: %s [--gpus G] [--allgather] [--quick]\n",
                  argv[0]);
      return 0;
    }
  }
  int avail = 0;
  CUDA_CHECK(cudaGetDeviceCount(&avail));
  if (gpus <= 0 || gpus > avail) gpus = avail;
  auto caps = init_device();
  const double peak = peak_tflops(caps, B200_DT_E4M3);
  std::printf("  GPUs used             : %d\n", gpus);

  // ---- CHECK: small fp16 problem split over the GPUs, gathered on the host ----
  bool ok = true;
  {
    const int64_t m = 512, n = 512 * gpus, k = 1024;
    auto fa = hopper::make_random_vector(size_t(m * k), 601, -1.f, 1.f);
    auto fb = hopper::make_random_vector(size_t(n * k), 602, -1.f, 1.f);
    auto ha = to_f16(fa), hb = to_f16(fb);
    auto ref = host_gemm(to_float(ha), to_float(hb), m, n, k);
    std::vector<float> got(size_t(m * n));
    std::vector<std::thread> th;
    std::mutex mu;
    for (int g = 0; g < gpus; ++g)
      th.emplace_back([&, g] {
        CUDA_CHECK(cudaSetDevice(g));
        auto [n0, n1] = shard_columns(n, gpus, g);
        void *dA, *dB, *dC;
        CUDA_CHECK(cudaMalloc(&dA, size_t(m * k) * 2));
        CUDA_CHECK(cudaMalloc(&dB, size_t((n1 - n0) * k) * 2 + 16));
        CUDA_CHECK(cudaMalloc(&dC, size_t(m * (n1 - n0)) * 2 + 16));
        CUDA_CHECK(cudaMemcpy(dA, ha.data(), size_t(m * k) * 2, cudaMemcpyHostToDevice));
        CUDA_CHECK(cudaMemcpy(dB, hb.data() + n0 * k, size_t((n1 - n0) * k) * 2, cudaMemcpyHostToDevice));
        run_checked(args_for(B200_DT_F16, B200_DT_F16, m, n1 - n0, k, dA, dB, dC, B200_VARIANT_AUTO));
        auto c = download_c(dC, B200_DT_F16, size_t(m * (n1 - n0)));
        std::lock_guard<std::mutex> lk(mu);
        for (int64_t r = 0; r < m; ++r)
          for (int64_t j = 0; j < n1 - n0; ++j) got[size_t(r * n + n0 + j)] = c[size_t(r * (n1 - n0) + j)];
        cudaFree(dA);
        cudaFree(dB);
        cudaFree(dC);
      });
    for (auto& t : th) t.join();
    auto rep = hopper::check_close(got, ref, 1e-2, 1e-2 * rms(ref));
    hopper::print_report(rep, "N-sharded fp16 vs host");
    ok = rep.pass;
  }
  if (!ok) return 1;

  // ---- GEMM: e4m3 16384 x 65536 x 8192, N split over the GPUs ----
  std::vector<Shard> sh(static_cast<size_t>(gpus));
  std::vector<ncclComm_t> comms(static_cast<size_t>(gpus));
  std::vector<int> devs(static_cast<size_t>(gpus));
  for (int g = 0; g < gpus; ++g) devs[size_t(g)] = g;
  if (allgather) NCCL_CHECK(ncclCommInitAll(comms.data(), gpus, devs.data()));
  std::barrier sync_point(gpus);
  const int warmup = 3, reps = 10;
  std::vector<double> ag_ms(size_t(gpus), 0.0), rl_ms(size_t(gpus), 0.0);
  std::vector<std::thread> th;
  for (int g = 0; g < gpus; ++g)
    th.emplace_back([&, g] {
      Shard& s = sh[size_t(g)];
      s.dev = g;
      CUDA_CHECK(cudaSetDevice(g));
      CUDA_CHECK(cudaStreamCreateWithFlags(&s.s, cudaStreamNonBlocking));
      std::tie(s.n0, s.n1) = shard_columns(N, gpus, g);
      const int64_t ng = s.n1 - s.n0;
      float* tmp = nullptr;
      CUDA_CHECK(cudaMalloc(&tmp, size_t(std::max(M, ng) * K) * 4));
      CUDA_CHECK(cudaMalloc(&s.dA, size_t(M * K)));
      CUDA_CHECK(cudaMalloc(&s.dB, size_t(ng * K)));
      CUDA_CHECK(cudaMalloc(&s.dC, size_t(M * ng) * 2));
      CUDA_CHECK(cudaMalloc(&s.sa, 4));
      CUDA_CHECK(cudaMalloc(&s.sb, 4));
      fill_uniform<<<1184, 256, 0, s.s>>>(tmp, M * K, 905);  // A is the same on every GPU
      B200_CHECK(b200_quantize_e4m3(tmp, M * K, s.dA, s.sa, s.s));
      fill_uniform<<<1184, 256, 0, s.s>>>(tmp, ng * K, 906 + uint64_t(s.n0));
      B200_CHECK(b200_quantize_e4m3(tmp, ng * K, s.dB, s.sb, s.s));
      CUDA_CHECK(cudaStreamSynchronize(s.s));
      cudaFree(tmp);
      auto a = args_for(B200_DT_E4M3, B200_DT_BF16, M, ng, K, s.dA, s.dB, s.dC, B200_VARIANT_AUTO);
      a.scale_a = s.sa;
      a.scale_b = s.sb;
      for (int i = 0; i < warmup; ++i) B200_CHECK(b200_gemm(&a, s.s));
      CUDA_CHECK(cudaStreamSynchronize(s.s));
      cudaEvent_t e0, e1;
      CUDA_CHECK(cudaEventCreate(&e0));
      CUDA_CHECK(cudaEventCreate(&e1));
      sync_point.arrive_and_wait();  // all GPUs start together
      CUDA_CHECK(cudaEventRecord(e0, s.s));
      for (int i = 0; i < reps; ++i) B200_CHECK(b200_gemm(&a, s.s));
      CUDA_CHECK(cudaEventRecord(e1, s.s));
      CUDA_CHECK(cudaEventSynchronize(e1));
      float ms = 0.f;
      CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
      s.ms = double(ms) / reps;
      uint32_t bits = 0;
      if (b200_gemm_status(s.s, 1, &bits) != B200_OK) {
        std::fprintf(stderr, "GPU %d: device status 0x%x\n", g, bits);
        std::exit(EXIT_FAILURE);
      }
      if (allgather) {
        void* gathered = nullptr;
        void* rowmajor = nullptr;
        CUDA_CHECK(cudaMalloc(&gathered, size_t(M * ng) * 2 * size_t(gpus)));
        CUDA_CHECK(cudaMalloc(&rowmajor, size_t(M * ng) * 2 * size_t(gpus)));
        sync_point.arrive_and_wait();
        CUDA_CHECK(cudaEventRecord(e0, s.s));
        NCCL_CHECK(ncclAllGather(s.dC, gathered, size_t(M * ng) * 2, ncclUint8, comms[size_t(g)], s.s));
        CUDA_CHECK(cudaEventRecord(e1, s.s));
        CUDA_CHECK(cudaEventSynchronize(e1));
        CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
        ag_ms[size_t(g)] = ms;
        CUDA_CHECK(cudaEventRecord(e0, s.s));
        relayout<<<1184, 256, 0, s.s>>>(static_cast<const uint4*>(gathered), static_cast<uint4*>(rowmajor), gpus, M,
                                        ng * 2 / 16);
        CUDA_CHECK(cudaEventRecord(e1, s.s));
        CUDA_CHECK(cudaEventSynchronize(e1));
        CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
        rl_ms[size_t(g)] = ms;
        cudaFree(gathered);
        cudaFree(rowmajor);
      }
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
    });
  for (auto& t : th) t.join();
  double max_ms = 0.0;
  for (const Shard& s : sh) max_ms = std::max(max_ms, s.ms);
  const double flops = 2.0 * double(M) * double(N) * double(K);
  const double tf = hopper::tflops(flops, max_ms);
  std::printf("\n[GEMM  ] e4m3 %lldx%lldx%lld, N split over %d GPU(s)\n", (long long)M, (long long)N, (long long)K, gpus);
  for (const Shard& s : sh)
    std::printf("  GPU %d: columns [%lld, %lld)  %.3f ms  %.2f TFLOPS\n", s.dev, (long long)s.n0, (long long)s.n1,
                s.ms, hopper::tflops(2.0 * double(M) * double(s.n1 - s.n0) * double(K), s.ms));
  char tag[64];
  std::snprintf(tag, sizeof(tag), "box (%d GPU) max-over-GPUs", gpus);
  print_bench(tag, max_ms, flops);
  std::printf("  %% of %d x dense e4m3 peak: %.1f%%\n", gpus, 100.0 * tf / (peak * gpus));
  if (allgather) {
    double ag = 0, rl = 0;
    for (int g = 0; g < gpus; ++g) {
      ag = std::max(ag, ag_ms[size_t(g)]);
      rl = std::max(rl, rl_ms[size_t(g)]);
    }
    const double bytes = double(M) * double(N) * 2.0;
    std::printf("  all-gather of C (%.2f GB): %.3f ms (%.0f GB/s per GPU in), re-layout %.3f ms\n", bytes / 1e9, ag,
                bytes * (gpus - 1) / gpus / (ag * 1e6), rl);
    for (auto c : comms) ncclCommDestroy(c);
  }
  hopper::CsvWriter csv("results/gemm_multi_gpu.csv",
                        {"gpus", "M", "N", "K", "max_ms", "tflops", "pct_peak", "allgather_ms", "relayout_ms"});
  double ag = 0, rl = 0;
  for (int g = 0; g < gpus; ++g) {
    ag = std::max(ag, ag_ms[size_t(g)]);
    rl = std::max(rl, rl_ms[size_t(g)]);
  }
  csv.row({std::to_string(gpus), std::to_string(M), std::to_string(N), std::to_string(K), std::to_string(max_ms),
           std::to_string(tf), std::to_string(tf / (peak * gpus)), std::to_string(ag), std::to_string(rl)});
  for (Shard& s : sh) {
    cudaSetDevice(s.dev);
    cudaFree(s.dA);
    cudaFree(s.dB);
    cudaFree(s.dC);
    cudaFree(s.sa);
    cudaFree(s.sb);
    cudaStreamDestroy(s.s);
  }
  return 0;
}
