// noalloc.cu — b200_gemm_noalloc: the GEMM entry point that allocates no device memory.
//
// Who needs it. b200_gemm allocates one 256-byte device status word with cudaMalloc
// on its first call on each device. Some callers cannot let a library do that:
// code running inside a framework that owns every device allocation through its
// own pool allocator (a stray cudaMalloc bypasses the pool's accounting and limits),
// processes that must keep their device footprint fixed after start-up (serving
// processes sized to share a GPU), and code that must not take the allocator's locks
// or synchronising calls on its path. This entry point runs the same kernel with
// its scratch in statically allocated device memory instead.
//
// Scratch. The GEMM kernel's only scratch is the status word its bounded waits
// write when one of them gives up. Here it lives in g_noalloc_scratch below: a
// file-scope `static __device__` array of kScratchBytes = 256 bytes, of which a call
// uses one 32-bit word. Every GPU that loads this library holds the array until
// the process exits. Requests that would need more scratch than the array holds
// are rejected with B200_ERR_SCRATCH_LIMIT: the GEMM needs one word for every
// shape, but the stream-K variant also needs a 32 MB partial-tile workspace, so an
// explicit stream-K request is rejected and AUTO never chooses it here.
//
// Sharing. All calls on a device share the one array, and it keeps whatever the
// last call left in it: each call clears its status word (a stream-ordered memset)
// before its kernel runs. Calls whose work overlaps on the GPU (different streams,
// or different host threads) race on that word: one call's clear can hide another
// call's failure report. Serialise the calls (one stream) when the status matters.
//
// Set-up. The first call on a device, with that device current, resolves the
// driver's tensor-map encoder and looks up the array's device address with
// cudaGetSymbolAddress (in host code the array's name is only a host-side stand-in;
// the kernel must be given the device address). Make that first call before any
// stream capture starts. Later calls only read the cached address.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>

#include "b200gemm.h"
#include "gemm_internal.h"

namespace {

constexpr size_t kScratchBytes = 256;
// Statically allocated device scratch of the allocation-free entry point.
static __device__ __align__(256) uint32_t g_noalloc_scratch[kScratchBytes / sizeof(uint32_t)];

std::mutex g_mu;
// Device address of g_noalloc_scratch, per device. Published with a release store
// after g_sms and g_cc_major are written and read with an acquire load, so a thread
// that finds the address also finds the SM count it needs to pick a variant.
std::atomic<uint32_t*> g_scratch_dev[64];
int g_sms[64] = {0};
int g_cc_major[64] = {0};

// Once per device, with `dev` current: everything the launch needs, no allocation.
int setup_device(int dev) {
  if (g_scratch_dev[dev].load(std::memory_order_acquire)) return B200_OK;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_dev[dev].load(std::memory_order_relaxed)) return B200_OK;
  int rc = b200::gemm_resolve_driver();
  if (rc != B200_OK) return rc;
  int sms = 0, major = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return B200_ERR_CUDA;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return B200_ERR_CUDA;
  void* ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr)
    return B200_ERR_CUDA;
  g_sms[dev] = sms;
  g_cc_major[dev] = major;
  g_scratch_dev[dev].store(static_cast<uint32_t*>(ptr), std::memory_order_release);
  return B200_OK;
}

// Scratch a call needs: the kernel's status word; the stream-K schedule also needs
// its partial-tile workspace (one 128 x 256 fp32 region per CTA), far more than
// the static array holds, so that variant is refused here (AUTO never picks it).
size_t scratch_bytes_needed(const B200GemmArgs& a) {
  if (a.variant == B200_VARIANT_2CTA_STREAMK) return sizeof(uint32_t) + size_t(256) * 128 * 256 * 4;
  return sizeof(uint32_t);
}

}  // namespace

extern "C" int b200_gemm_noalloc(const B200GemmArgs* args, void* stream_v, int check_status) {
  int rc = b200::gemm_validate(args);
  if (rc != B200_OK) return rc;
  const B200GemmArgs& a = *args;
  if (a.M == 0 || a.N == 0) return B200_OK;
  if (scratch_bytes_needed(a) > kScratchBytes) return B200_ERR_SCRATCH_LIMIT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return B200_ERR_CUDA;
  rc = setup_device(dev);
  if (rc != B200_OK) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  uint32_t* status = g_scratch_dev[dev].load(std::memory_order_acquire);
  // The array keeps the previous call's value: start this call's word at zero.
  if (cudaMemsetAsync(status, 0, sizeof(uint32_t), stream) != cudaSuccess) return B200_ERR_CUDA;
  rc = b200::gemm_launch_impl(a, stream, g_sms[dev], g_cc_major[dev], status, /*allow_workspace=*/false);
  if (rc != B200_OK || !check_status) return rc;
  // Optional synchronous check of this call's status word (no allocation either).
  if (cudaStreamSynchronize(stream) != cudaSuccess) return B200_ERR_CUDA;
  uint32_t v = 0;
  if (cudaMemcpy(&v, status, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return B200_ERR_CUDA;
  return v ? B200_ERR_DEVICE_TIMEOUT : B200_OK;
}
