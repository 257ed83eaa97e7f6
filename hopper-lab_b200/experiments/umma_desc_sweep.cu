// umma_desc_sweep — field-by-field check of the tcgen05 shared-memory and instruction
// descriptors the GEMM kernels use (sdesc_k_sw128, idesc_f32acc in sm100_ptx.cuh).
//
// B200 counterpart of the reference's descriptor probes (src/04_wgmma/wgmma_swizzle128.cu:112-127
// sweeps the wgmma base_offset 0..7 and reports which values PASS; src/07_fp8/wgmma_fp8.cu:143-154
// repeats it for e4m3). A GEMM that fails cannot say which descriptor field is wrong;
// one tcgen05.mma tile can. One CTA stages an A tile (128 rows x one 128-byte K atom)
// and a B tile (N rows x one atom) in shared memory in the 128-byte-swizzled K-major
// layout a TMA SWIZZLE_128B load produces (written here by plain stores:
// 16-byte chunk j of row r goes to r*128 + ((j ^ (r & 7)) << 4)), issues `steps` MMAs
// of 32 bytes of K each with the descriptor under test, reads D back from TMEM and
// compares it with a host GEMM over the same K.
//
// Sweeps (each line: the field value, PASS/fail, max |error|):
//   base_offset 0..7              (shared-memory descriptor bits 49-51)
//   swizzle mode 0/2/4/6          (bits 61-63: none, 128B, 64B, 32B)
//   stride byte offset 512/1024/2048 for A (bits 32-45: 8-row group pitch)
//   A leading byte offset 16/32/1024 (bits 16-29; unused for swizzled K-major tiles)
//   K steps 1..4                  (start address + 32 bytes per step inside the atom)
//   N 64/128/192/256              (instruction descriptor bits 17-22)
//   A/B format f16, bf16, e4m3    (instruction descriptor bits 7-12 and the kind)
// Every value keeps all shared-memory reads inside the staged buffers: the largest
// A pitch (2048 bytes) reaches 31 KB of the 32 KB A region, the unswizzled layout of
// a 256-row B tile 31.3 KB of the 32 KB B region, and 4 KB of slack follow. The library's own
// descriptor is the base case of every sweep; the [CHECK ] lines assert that it
// passes and that the values the kernels rely on are the only passing ones where a
// field matters.
#include "exp_common.h"
#include "sm100_ptx.cuh"

using namespace exp_common;

namespace {

constexpr uint32_t kThreads = 128;
constexpr uint32_t kARegion = 32768;  // A tile + room for the widest stride sweep
constexpr uint32_t kBRegion = 32768;  // 256 rows x 128 bytes

struct Probe {
  uint32_t n = 256;        // MMA N
  uint32_t steps = 4;      // 32-byte K steps (1..4)
  uint32_t base_off = 0;   // descriptor base offset field
  uint32_t swz = 2;        // swizzle mode field
  uint32_t a_sbo = 1024;   // A stride byte offset
  uint32_t lbo = 16;       // A leading byte offset (B keeps 16)
};

__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t base_off,
                                              uint32_t swz) {
  // The library's descriptor with every field under test replaced.
  uint64_t d = b200::sdesc_k_sw128(saddr);
  d &= ~(uint64_t(0x3FFFu) << 16);
  d &= ~(uint64_t(0x3FFFu) << 32);
  d &= ~(uint64_t(0x7u) << 49);
  d &= ~(uint64_t(0x7u) << 61);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(base_off & 0x7u) << 49;
  d |= uint64_t(swz & 0x7u) << 61;
  return d;
}

template <int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    probe_kernel(const uint8_t* A, const uint8_t* B, float* D, Probe pr, uint32_t idesc, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_slot;
  const uint32_t raw = b200::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* basep = smem_raw + (base - raw);
  // zero both regions, then stage the tiles in the 128-byte-swizzled layout
  for (uint32_t i = threadIdx.x; i < (kARegion + kBRegion) / 16u; i += blockDim.x)
    reinterpret_cast<uint4*>(basep)[i] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < 128u * 8u; i += blockDim.x) {
    const uint32_t r = i / 8u, j = i % 8u;
    *reinterpret_cast<uint4*>(basep + r * 128u + ((j ^ (r & 7u)) << 4)) =
        reinterpret_cast<const uint4*>(A)[i];
  }
  for (uint32_t i = threadIdx.x; i < pr.n * 8u; i += blockDim.x) {
    const uint32_t r = i / 8u, j = i % 8u;
    *reinterpret_cast<uint4*>(basep + kARegion + r * 128u + ((j ^ (r & 7u)) << 4)) =
        reinterpret_cast<const uint4*>(B)[i];
  }
  const uint32_t bar_a = b200::smem_u32(&bar);
  if (threadIdx.x == 0) {
    b200::mbar_init(bar_a, 1);
    b200::fence_mbar_init();
  }
  b200::fence_proxy_async_shared();  // generic stores -> visible to the tensor core
  if (threadIdx.x < 32) {
    b200::tmem_alloc<1>(b200::smem_u32(&tmem_slot), 256);
    b200::tmem_relinquish<1>();
  }
  b200::tc_fence_before();
  __syncthreads();
  b200::tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0) {
    for (uint32_t k = 0; k < pr.steps; ++k) {
      const uint64_t da = make_desc(base + 32u * k, pr.lbo, pr.a_sbo, pr.base_off, pr.swz);
      const uint64_t db = make_desc(base + kARegion + 32u * k, 16u, 1024u, pr.base_off, pr.swz);
      b200::umma<1, KIND>(tmem, da, db, idesc, k != 0u ? 1u : 0u);
    }
    b200::umma_commit<1>(bar_a);
    if (!b200::mbar_wait_bounded(bar_a, 0, 1000000000ull)) atomicOr(status, 1u);
  }
  __syncthreads();
  b200::tc_fence_after();
  // warp w reads TMEM lanes 32w..32w+31 (rows of D), 32 columns at a time
  const uint32_t w = threadIdx.x / 32u, row = threadIdx.x;
  for (uint32_t c0 = 0; c0 < pr.n; c0 += 32u) {
    uint32_t v[32];
    b200::tmem_ld_x32(tmem + ((32u * w) << 16) + c0, v);
    b200::tmem_wait_ld();
    for (uint32_t i = 0; i < 32u; ++i) D[size_t(row) * pr.n + c0 + i] = __uint_as_float(v[i]);
  }
  b200::tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    b200::tc_fence_after();
    b200::tmem_dealloc<1>(tmem, 256);
  }
}

struct Tiles {
  int ab;                       // B200_DT_*
  std::vector<uint8_t> a, b;    // raw element bytes: 128 x 128 B and 256 x 128 B
  std::vector<float> af, bf;    // their fp32 values
  uint32_t elems;               // elements per 128-byte row
};

Tiles make_tiles(int ab) {
  Tiles t;
  t.ab = ab;
  t.elems = ab == B200_DT_E4M3 ? 128u : 64u;
  auto ha = hopper::make_random_vector(size_t(128) * t.elems, 311, -1.f, 1.f);
  auto hb = hopper::make_random_vector(size_t(256) * t.elems, 312, -1.f, 1.f);
  auto pack = [&](const std::vector<float>& h, std::vector<uint8_t>& bytes, std::vector<float>& vals) {
    bytes.resize(h.size() * (ab == B200_DT_E4M3 ? 1 : 2));
    if (ab == B200_DT_F16) {
      auto v = to_f16(h);
      std::memcpy(bytes.data(), v.data(), bytes.size());
      vals = to_float(v);
    } else if (ab == B200_DT_BF16) {
      auto v = to_bf16(h);
      std::memcpy(bytes.data(), v.data(), bytes.size());
      vals = to_float(v);
    } else {
      auto v = to_e4m3(h);
      std::memcpy(bytes.data(), v.data(), bytes.size());
      vals = to_float(v);
    }
  };
  pack(ha, t.a, t.af);
  pack(hb, t.b, t.bf);
  return t;
}

struct Outcome {
  bool pass;
  double max_abs;
};

Outcome run_probe(const Tiles& t, const Probe& pr) {
  const uint32_t kstep_elems = t.ab == B200_DT_E4M3 ? 32u : 16u;
  const uint32_t kused = pr.steps * kstep_elems;
  // host reference over the first kused elements of K (the reference's CHECK loop)
  std::vector<float> ref(size_t(128) * pr.n);
  for (uint32_t m = 0; m < 128; ++m)
    for (uint32_t n = 0; n < pr.n; ++n) {
      float acc = 0.f;
      for (uint32_t k = 0; k < kused; ++k) acc += t.af[size_t(m) * t.elems + k] * t.bf[size_t(n) * t.elems + k];
      ref[size_t(m) * pr.n + n] = acc;
    }
  hopper::DeviceBuffer<uint8_t> dA(t.a.size()), dB(t.b.size());
  hopper::DeviceBuffer<float> dD(ref.size());
  hopper::DeviceBuffer<uint32_t> dS(1);
  dA.upload(t.a);
  dB.upload(t.b);
  CUDA_CHECK(cudaMemset(dS.get(), 0, 4));
  const uint32_t fa = t.ab == B200_DT_BF16 ? 1u : 0u;
  const uint32_t idesc = b200::idesc_f32acc(fa, fa, 128u, pr.n);
  const size_t smem = 1024 + kARegion + kBRegion + 4096;
  if (t.ab == B200_DT_E4M3) {
    CUDA_CHECK(cudaFuncSetAttribute(reinterpret_cast<const void*>(probe_kernel<1>),
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    probe_kernel<1><<<1, kThreads, smem>>>(dA.get(), dB.get(), dD.get(), pr, idesc, dS.get());
  } else {
    CUDA_CHECK(cudaFuncSetAttribute(reinterpret_cast<const void*>(probe_kernel<0>),
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    probe_kernel<0><<<1, kThreads, smem>>>(dA.get(), dB.get(), dD.get(), pr, idesc, dS.get());
  }
  CUDA_CHECK_LAST();
  CUDA_CHECK(cudaDeviceSynchronize());
  uint32_t st = 0;
  CUDA_CHECK(cudaMemcpy(&st, dS.get(), 4, cudaMemcpyDeviceToHost));
  if (st) {
    std::fprintf(stderr, "probe wait timed out\n");
    std::exit(EXIT_FAILURE);
  }
  auto rep = hopper::check_close(dD.download(), ref, 1e-3, 1e-3);
  return {rep.pass, rep.max_abs_err};
}

const char* dt_name(int ab) { return ab == B200_DT_F16 ? "f16" : ab == B200_DT_BF16 ? "bf16" : "e4m3"; }

int g_fail = 0;

void check(bool ok, const char* what) {
  std::printf("[CHECK ] %-58s : %s\n", what, ok ? "PASS" : "FAIL");
  if (!ok) g_fail = 1;
}

void line(hopper::CsvWriter& csv, const char* field, const std::string& value, int ab, const Outcome& o) {
  std::printf("  %-14s %-6s %-5s : %s (max_abs=%.3e)\n", field, value.c_str(), dt_name(ab), o.pass ? "PASS" : "fail",
              o.max_abs);
  csv.row({field, value, dt_name(ab), o.pass ? "pass" : "fail", std::to_string(o.max_abs)});
}

}  // namespace

int main(int argc, char** argv) {
  const Opts o = parse(argc, argv, "umma_desc_sweep: tcgen05 descriptor fields, one MMA tile (04_wgmma / 07_fp8 probes)");
  (void)o;
  init_device();
  hopper::CsvWriter csv("results/umma_desc_sweep.csv", {"field", "value", "dtype", "result", "max_abs"});
  const Tiles f16 = make_tiles(B200_DT_F16);

  std::printf("\n[SWEEP  ] base_offset (bits 49-51), f16, N=256, 4 K steps\n");
  int passing_base = 0, base0 = 0;
  for (uint32_t v = 0; v < 8; ++v) {
    Probe pr;
    pr.base_off = v;
    const Outcome r = run_probe(f16, pr);
    line(csv, "base_offset", std::to_string(v), B200_DT_F16, r);
    passing_base += r.pass;
    if (v == 0) base0 = r.pass;
  }
  check(base0, "base_offset 0 (1024-byte aligned atoms) passes");

  std::printf("\n[SWEEP  ] swizzle mode (bits 61-63), f16\n");
  bool swz_ok = true;
  for (uint32_t v : {0u, 2u, 4u, 6u}) {
    Probe pr;
    pr.swz = v;
    const Outcome r = run_probe(f16, pr);
    line(csv, "swizzle", std::to_string(v), B200_DT_F16, r);
    swz_ok &= (r.pass == (v == 2u));
  }
  check(swz_ok, "only swizzle mode 2 (128-byte) matches the TMA layout");

  std::printf("\n[SWEEP  ] A stride byte offset (bits 32-45), f16\n");
  bool sbo_ok = true;
  for (uint32_t v : {512u, 1024u, 2048u}) {
    Probe pr;
    pr.a_sbo = v;
    const Outcome r = run_probe(f16, pr);
    line(csv, "a_sbo", std::to_string(v), B200_DT_F16, r);
    sbo_ok &= (r.pass == (v == 1024u));
  }
  check(sbo_ok, "only SBO = 1024 bytes (8 rows x 128 B) passes");

  std::printf("\n[SWEEP  ] leading byte offset (bits 16-29), f16\n");
  bool lbo_ok = true;
  for (uint32_t v : {16u, 32u, 1024u}) {
    Probe pr;
    pr.lbo = v;
    const Outcome r = run_probe(f16, pr);
    line(csv, "lbo", std::to_string(v), B200_DT_F16, r);
    lbo_ok &= r.pass;
  }
  check(lbo_ok, "LBO is ignored for swizzled K-major tiles");

  std::printf("\n[SWEEP  ] K steps (start address + 32 B per step), N (idesc bits 17-22), format\n");
  bool k_ok = true, n_ok = true, fmt_ok = true;
  for (uint32_t v = 1; v <= 4; ++v) {
    Probe pr;
    pr.steps = v;
    const Outcome r = run_probe(f16, pr);
    line(csv, "k_steps", std::to_string(v), B200_DT_F16, r);
    k_ok &= r.pass;
  }
  for (uint32_t v : {64u, 128u, 192u, 256u}) {
    Probe pr;
    pr.n = v;
    const Outcome r = run_probe(f16, pr);
    line(csv, "n", std::to_string(v), B200_DT_F16, r);
    n_ok &= r.pass;
  }
  for (int ab : {B200_DT_BF16, B200_DT_E4M3}) {
    const Tiles t = make_tiles(ab);
    for (uint32_t steps : {1u, 4u}) {
      Probe pr;
      pr.steps = steps;
      const Outcome r = run_probe(t, pr);
      line(csv, "format_steps", std::to_string(steps), ab, r);
      fmt_ok &= r.pass;
    }
  }
  check(k_ok, "every 32-byte K step inside the 128-byte atom");
  check(n_ok, "N = 64 / 128 / 192 / 256 in the instruction descriptor");
  check(fmt_ok, "bf16 and e4m3 formats (kind::f16, kind::f8f6f4)");
  std::printf("  base_offset values passing: %d of 8\n", passing_base);
  return g_fail ? 1 : 0;
}
