// dsmem_copy — shared-memory to shared-memory streaming between the two CTA pairs of a
// 4-CTA cluster, the transport the B-sharing GEMM variant (SCHED_SHARE) forwards its B
// rows over. Counterpart of the reference's DSMEM probes (src/06_cluster), measured for
// the question that variant raises: can one SM forward 16 KB per pipeline stage
// (about 25 GB/s at the f16 MMA rate) to another SM of its GPC?
//
// Grid = SM count, regular clusters of 2, preferred clusters of 4 (where a GPC has room).
// In every 4-CTA cluster, CTA r streams CHUNK-byte chunks into CTA r^2 through a ring of
// four slots: one `cp.async.bulk.shared::cluster.shared::cta` per chunk ("bulk") or a
// warp of 16-byte `st.shared::cluster` stores ("warp"). The receiver waits for each chunk
// on an mbarrier and hands the slot back with a remote arrive. Every wait is bounded.
// A CHECK line verifies the received bytes of the last ring pass.
#include "exp_common.h"
#include "sm100_ptx.cuh"

using namespace exp_common;

namespace {

constexpr int kSlots = 4;
constexpr uint64_t kWaitNs = 200000000ull;  // 0.2 s per wait

__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, uint64_t t0) {
  while (!b200::mbar_try_wait(bar, parity)) {
    if (b200::globaltimer_ns() - t0 > kWaitNs) return false;
  }
  return true;
}

// out[4*block]: cluster size, ns for the stream (receiver), ok, bad-word count
__global__ void __launch_bounds__(128, 1)
    stream_kernel(unsigned long long* out, int mode, int chunk, int iters) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t nct = b200::cluster_nctarank(), crank = b200::cluster_ctarank();
  const uint32_t raw = b200::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* basep = smem_raw + (base - raw);
  const uint32_t bar_full = base, bar_free = base + 64;
  const uint32_t send = base + 1024, recv = send + kSlots * chunk;
  uint32_t* send_w = reinterpret_cast<uint32_t*>(basep + 1024);
  uint32_t* recv_w = reinterpret_cast<uint32_t*>(basep + 1024 + kSlots * chunk);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t words = uint32_t(kSlots * chunk / 4);
  for (uint32_t i = threadIdx.x; i < words; i += blockDim.x) {
    send_w[i] = (blockIdx.x << 20) ^ i;
    recv_w[i] = 0u;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      b200::mbar_init(bar_full + 8 * s, 1);
      b200::mbar_init(bar_free + 8 * s, 1);
    }
    b200::fence_mbar_init();
  }
  b200::fence_proxy_async_shared();
  __syncthreads();
  b200::cluster_sync();
  const unsigned long long t_start = b200::globaltimer_ns();
  unsigned long long t_end = 0;
  uint32_t ok = 1;
  if (nct == 4) {
    const uint32_t peer = crank ^ 2u;
    const uint64_t t0 = b200::globaltimer_ns();
    if (warp == 0) {
      for (int i = 0; i < iters && ok; ++i) {
        const int s = i % kSlots;
        const uint32_t ph = uint32_t(i / kSlots) & 1u;
        if (lane == 0) ok = wait_phase(bar_free + 8 * s, ph ^ 1u, t0) ? 1u : 0u;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        const uint32_t src = send + s * chunk, dst = b200::mapa_shared(recv + s * chunk, peer);
        const uint32_t rbar = b200::mapa_shared(bar_full + 8 * s, peer);
        if (mode == 0) {
          if (lane == 0) b200::bulk_copy_s2c(dst, src, uint32_t(chunk), rbar);
        } else {
          for (int off = int(lane) * 16; off < chunk; off += 32 * 16) {
            uint32_t a0, a1, a2, a3;
            b200::ld_shared_v4(src + off, a0, a1, a2, a3);
            b200::st_shared_cluster_v4(dst + off, a0, a1, a2, a3);
          }
          __syncwarp();
          if (lane == 0) b200::mbar_arrive_cluster(rbar);
        }
      }
    } else if (warp == 1 && lane == 0) {
      for (int i = 0; i < iters && ok; ++i) {
        const int s = i % kSlots;
        const uint32_t ph = uint32_t(i / kSlots) & 1u;
        if (mode == 0) b200::mbar_arrive_expect_tx(bar_full + 8 * s, uint32_t(chunk));
        if (!wait_phase(bar_full + 8 * s, ph, t0)) {
          ok = 0;
          break;
        }
        b200::mbar_arrive_cluster(b200::mapa_shared(bar_free + 8 * s, peer));
      }
      t_end = b200::globaltimer_ns();
    }
  }
  __syncthreads();
  b200::cluster_sync();
  // every slot received at least once holds the sender's pattern
  uint32_t bad = 0;
  if (nct == 4 && iters >= kSlots) {
    const uint32_t sender = blockIdx.x - crank + (crank ^ 2u);
    for (uint32_t i = threadIdx.x; i < words; i += blockDim.x)
      if (recv_w[i] != ((sender << 20) ^ i)) ++bad;
  }
  atomicAdd(reinterpret_cast<unsigned long long*>(out + 4 * blockIdx.x + 3), (unsigned long long)bad);
  if (warp == 1 && lane == 0) {
    out[4 * blockIdx.x + 0] = nct;
    out[4 * blockIdx.x + 1] = t_end ? t_end - t_start : 0;
  }
  if (threadIdx.x == 0) out[4 * blockIdx.x + 2] = ok;
}

}  // namespace

int main(int argc, char** argv) {
  const Opts o = parse(argc, argv, "dsmem_copy: SM-to-SM streaming inside 4-CTA clusters (06_cluster)");
  auto caps = init_device();
  hopper::CsvWriter csv("results/dsmem_copy.csv",
                        {"mode", "chunk", "iters", "clusters4", "us_per_chunk", "gbs_per_sm", "tbs_total"});
  const int grid = caps.sm_count / 4 * 4;
  const int smem = 1024 + 2 * kSlots * 16384 + 1024;
  CUDA_CHECK(cudaFuncSetAttribute(stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  unsigned long long* d = nullptr;
  CUDA_CHECK(cudaMalloc(&d, sizeof(unsigned long long) * 4 * grid));
  const int iters = o.quick ? 200 : 2000;
  bool all_ok = true;
  for (int mode : {0, 1}) {
    for (int chunk : {4096, 16384}) {
      CUDA_CHECK(cudaMemset(d, 0, sizeof(unsigned long long) * 4 * grid));
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(grid);
      cfg.blockDim = dim3(128);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute at[2];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 2;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      at[1].id = cudaLaunchAttributePreferredClusterDimension;
      at[1].val.preferredClusterDim.x = 4;
      at[1].val.preferredClusterDim.y = 1;
      at[1].val.preferredClusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 2;
      CUDA_CHECK(cudaLaunchKernelEx(&cfg, stream_kernel, d, mode, chunk, iters));
      CUDA_CHECK(cudaDeviceSynchronize());
      std::vector<unsigned long long> h(size_t(4) * grid);
      CUDA_CHECK(cudaMemcpy(h.data(), d, h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
      double ns = 0;
      int n4 = 0;
      unsigned long long bad = 0, fails = 0;
      for (int b = 0; b < grid; ++b) {
        if (h[4 * b] != 4) continue;
        ++n4;
        ns += double(h[4 * b + 1]);
        bad += h[4 * b + 3];
        fails += h[4 * b + 2] ? 0 : 1;
      }
      if (n4 == 0) {
        std::printf("[CHECK ] no 4-CTA cluster was formed on this device\n");
        return EXIT_FAILURE;
      }
      ns /= n4;
      const double us_chunk = ns / 1e3 / iters;
      const double gbs = double(chunk) * iters / ns;
      const char* m = mode == 0 ? "bulk copy" : "warp st.shared::cluster";
      const bool pass = bad == 0 && fails == 0;
      all_ok = all_ok && pass;
      std::printf("[CHECK ] %-24s chunk %5d B: %s (%llu bad words, %llu timed-out CTAs)\n", m, chunk,
                  pass ? "PASS" : "FAIL", bad, fails);
      std::printf("[BENCH ] %-24s chunk %5d B: %.3f us/chunk  %.1f GB/s per SM  %.2f TB/s over %d CTAs in %d clusters of 4\n",
                  m, chunk, us_chunk, gbs, gbs * n4 / 1e3, n4, n4 / 4);
      csv.row({mode == 0 ? "bulk" : "warp", std::to_string(chunk), std::to_string(iters), std::to_string(n4 / 4),
               std::to_string(us_chunk), std::to_string(gbs), std::to_string(gbs * n4 / 1e3)});
    }
  }
  cudaFree(d);
  return all_ok ? 0 : EXIT_FAILURE;
}
