// b200gemm.cu — the C ABI (include/b200gemm.h): validation, tensor-map encoding,
// variant selection and launch. Host code only; kernels live in inst_*.cu.
//
// Reference interfaces replaced here:
//   make_tmap_h / make_tmap_f           src/05_gemm/gemm_ws.cu:162-199
//   make_tmap_fp8                       src/07_fp8/gemm_fp8.cu:145-168
//   launch_config<S,tma> / dispatch     src/05_gemm/gemm_ws.cu:201-235
//   persistent launch_config (grid = min(tiles, SMs*occ))
//                                       src/08_persistent/gemm_fp8_persist.cu:222-242
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <new>

#include "b200gemm.h"
#include "gemm_internal.h"
#include "gemm_launch.cuh"

namespace {

using b200::GemmCfg;
using b200::KParams;
using b200::LaunchPlan;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

std::mutex g_mu;
// Per-device state, set up once. The pointers are published with release stores
// after every field they guard is written, and read with acquire loads on the fast
// path, so a thread that sees a pointer also sees the SM count and the rest.
//
// stream-K partial-tile workspace: one 128 x 256 fp32 region and one ready flag per
// CTA slot (256 slots cover any grid on a 148-SM part), allocated on first use
constexpr int kSkSlots = 256;
std::atomic<float*> g_sk_work[64];
uint32_t* g_sk_flags[64] = {nullptr};
std::atomic<uint32_t> g_sk_epoch[64];
// Stream-K launches on one device share that workspace, so they must not overlap on
// the GPU. Launches on one stream are ordered by the stream; a launch on another
// stream first waits (cudaStreamWaitEvent) for the event recorded after the previous
// stream-K launch. g_sk_mu serialises the bookkeeping (host only).
std::mutex g_sk_mu;
cudaEvent_t g_sk_event[64] = {nullptr};
cudaStream_t g_sk_last_stream[64] = {nullptr};
bool g_sk_recorded[64] = {false};

int streamk_workspace(int dev, float** work, uint32_t** flags) {
  float* w = g_sk_work[dev].load(std::memory_order_acquire);
  if (!w) {
    std::lock_guard<std::mutex> lk(g_mu);
    w = g_sk_work[dev].load(std::memory_order_relaxed);
    if (!w) {
      uint32_t* f = nullptr;
      cudaEvent_t ev = nullptr;
      if (cudaMalloc(&w, size_t(kSkSlots) * 128 * 256 * sizeof(float)) != cudaSuccess) return B200_ERR_CUDA;
      if (cudaMalloc(&f, size_t(kSkSlots) * sizeof(uint32_t)) != cudaSuccess) return B200_ERR_CUDA;
      if (cudaMemset(f, 0, size_t(kSkSlots) * sizeof(uint32_t)) != cudaSuccess) return B200_ERR_CUDA;
      if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return B200_ERR_CUDA;
      g_sk_flags[dev] = f;
      g_sk_event[dev] = ev;
      g_sk_work[dev].store(w, std::memory_order_release);
    }
  }
  *work = w;
  *flags = g_sk_flags[dev];
  return B200_OK;
}
EncodeTiledFn g_encode = nullptr;
std::atomic<uint32_t*> g_status[64];
int g_sm_count[64] = {0};
int g_cc_major[64] = {0};

constexpr uint64_t kDefaultWaitNs = 1000000000ull;  // 1 s per wait
// L2 cache policies of the operand loads and C stores (KParams::l2_policy bits): A
// evict_last, B evict_first, C stores evict_first. Under the 1 kW power cap the clock
// follows the energy of each GEMM, and these hints cut it. Sustained 8192^3, cuBLASLt
// interleaved in rounds (bench.py --mode power): e4m3 2665-2701 TFLOPS and 403-407 mJ
// per GEMM against 2578-2608 and 408-421 with evict_normal everywhere; f16 1305 TFLOPS
// and 832 mJ against 1287 and 877 (f16 reads more DRAM bytes with these hints, 1256 vs
// 884 MB per launch, yet spends less energy per GEMM).
#ifndef B200_L2_POLICY
#define B200_L2_POLICY 7u
#endif
constexpr uint32_t kL2Policy = B200_L2_POLICY;

// Experimental builds only (compiled with -DB200_EXPERIMENT_ENV, never by default):
// the L2 policy bits, the operand maps' L2 promotion (128 or 256 bytes) and the L2
// prefetch distance in k-blocks come from the environment variables B200_L2_POLICY,
// B200_L2_PROMO and B200_PREFETCH_K at every call, so that bench.py --mode power and
// --mode sweep can interleave these settings inside one process (an empty value keeps
// the library's own choice).
uint32_t l2_policy_bits(uint32_t dflt) {
#ifdef B200_EXPERIMENT_ENV
  if (const char* e = std::getenv("B200_L2_POLICY"); e && *e) return uint32_t(std::atoi(e));
#endif
  return dflt;
}
uint32_t prefetch_k_blocks(uint32_t dflt) {
#ifdef B200_EXPERIMENT_ENV
  if (const char* e = std::getenv("B200_PREFETCH_K"); e && *e) return uint32_t(std::atoi(e));
#endif
  return dflt;
}
CUtensorMapL2promotion l2_promotion() {
#ifdef B200_EXPERIMENT_ENV
  if (const char* e = std::getenv("B200_L2_PROMO"))
    if (std::atoi(e) == 256) return CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
#endif
  return CU_TENSOR_MAP_L2_PROMOTION_L2_128B;
}

constexpr int kDefaultGroupM = 8;
// 256x512 tiles are twice as wide, so twice as many block-rows per group keep a wave's
// A and B panels balanced: at 8192^3 under the power cap, 2-4 % less energy per GEMM
// than G = 8 (f16 828 vs 843 mJ, e4m3 423 vs 439) and 0.4-1 % more throughput.
constexpr int kDefaultGroupMWide = 16;

int resolve_encode() {
  if (g_encode) return B200_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e =
      cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return B200_ERR_CUDA;
  g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  return B200_OK;
}

// Per-device one-time set-up: driver entry point, SM count, status word.
int device_setup(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return B200_ERR_CUDA;
  if (dev < 0 || dev >= 64) return B200_ERR_CUDA;
  *dev_out = dev;
  if (g_status[dev].load(std::memory_order_acquire)) return B200_OK;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_status[dev].load(std::memory_order_relaxed)) return B200_OK;
  int rc = resolve_encode();
  if (rc != B200_OK) return rc;
  int sms = 0, major = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return B200_ERR_CUDA;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return B200_ERR_CUDA;
  uint32_t* st = nullptr;
  if (cudaMalloc(&st, 256) != cudaSuccess) return B200_ERR_CUDA;
  if (cudaMemset(st, 0, 256) != cudaSuccess) return B200_ERR_CUDA;
  g_sm_count[dev] = sms;
  g_cc_major[dev] = major;
  g_status[dev].store(st, std::memory_order_release);
  return B200_OK;
}

uint32_t* status_word(int dev) { return g_status[dev].load(std::memory_order_acquire); }

int elem_bytes(int dt) {
  switch (dt) {
    case B200_DT_F16:
    case B200_DT_BF16: return 2;
    case B200_DT_E4M3: return 1;
    case B200_DT_F32: return 4;
    default: return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 2D tensor map over a row-major [rows x cols] matrix with leading dimension ld
// (elements), box [box_rows x box_cols], 128-byte swizzle. Out-of-range boxes are
// zero-filled on load and clipped on store, which is what makes ragged M/N/K work.
int encode_2d(CUtensorMap* m, const void* ptr, int dt, uint64_t rows, uint64_t cols, uint64_t ld,
              uint32_t box_rows, uint32_t box_cols) {
  CUtensorMapDataType t;
  switch (dt) {
    case B200_DT_F16: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    case B200_DT_BF16: t = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    case B200_DT_E4M3: t = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
    case B200_DT_F32: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    default: return B200_ERR_INVALID_ARG;
  }
  const cuuint64_t gdim[2] = {cols, rows};
  const cuuint64_t gstride[1] = {ld * static_cast<uint64_t>(elem_bytes(dt))};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  std::memset(m, 0, sizeof(*m));
  CUresult r = g_encode(m, t, 2, const_cast<void*>(ptr), gdim, gstride, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        l2_promotion(), CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_TMAP;
}

struct VariantShape {
  int cg, sched, tn;
  uint32_t tile_m, tile_n, max_stages, default_stages, atoms;
};

// Tile and ring facts of one kernel configuration. Stage bytes do not depend on
// the element type (one 128-byte K atom per row), so the f16 instantiation's
// constants stand for every dtype.
template <int CG, int SCHED, int TN>
void fill_shape(VariantShape* vs) {
  using Cfg = GemmCfg<b200::DT_F16, b200::DT_F16, CG, SCHED, TN>;
  vs->cg = CG;
  vs->sched = SCHED;
  vs->tn = TN;
  vs->tile_m = uint32_t(Cfg::BM * CG);
  vs->tile_n = uint32_t(Cfg::BN);
  vs->max_stages = Cfg::MAX_STAGES;
  vs->default_stages = Cfg::MAX_STAGES;
  vs->atoms = uint32_t(Cfg::ATOMS);
}

template <int CG, int TN>
uint32_t shape_smem(uint32_t stages) {
  return GemmCfg<b200::DT_F16, b200::DT_F16, CG, b200::SCHED_STATIC, TN>::smem_bytes(stages);
}

// Tile widths: 1-CTA variants 256; pairs 128, 256 or 512 (stream-K 128 or 256).
// `tile_n` 0 picks the variant's default width (256).
int variant_shape(int variant, int tile_n, VariantShape* vs) {
  if (tile_n != 0 && tile_n != 128 && tile_n != 256 && tile_n != 512) return B200_ERR_INVALID_ARG;
  const int tn = tile_n ? tile_n : 256;
  switch (variant) {
    case B200_VARIANT_1CTA:
    case B200_VARIANT_PERSISTENT:
      if (tn != 256) return B200_ERR_INVALID_ARG;
      fill_shape<1, b200::SCHED_STATIC, 256>(vs);
      break;
    case B200_VARIANT_CLC:
      if (tn != 256) return B200_ERR_INVALID_ARG;
      fill_shape<1, b200::SCHED_CLC, 256>(vs);
      break;
    case B200_VARIANT_2CTA:
      if (tn == 128) fill_shape<2, b200::SCHED_STATIC, 128>(vs);
      else if (tn == 256) fill_shape<2, b200::SCHED_STATIC, 256>(vs);
      else fill_shape<2, b200::SCHED_STATIC, 512>(vs);
      break;
    case B200_VARIANT_2CTA_CLC:
      if (tn == 128) fill_shape<2, b200::SCHED_CLC, 128>(vs);
      else if (tn == 256) fill_shape<2, b200::SCHED_CLC, 256>(vs);
      else fill_shape<2, b200::SCHED_CLC, 512>(vs);
      break;
    case B200_VARIANT_2CTA_STREAMK:
      if (tn == 512) return B200_ERR_INVALID_ARG;
      if (tn == 128) fill_shape<2, b200::SCHED_STREAMK, 128>(vs);
      else fill_shape<2, b200::SCHED_STREAMK, 256>(vs);
      break;
    default: return B200_ERR_INVALID_ARG;
  }
  return B200_OK;
}

uint32_t variant_smem(const VariantShape& vs, uint32_t stages) {
  if (vs.cg == 1) return shape_smem<1, 256>(stages);
  if (vs.tn == 128) return shape_smem<2, 128>(stages);
  if (vs.tn == 256) return shape_smem<2, 256>(stages);
  return shape_smem<2, 512>(stages);
}

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// L2 prefetch distance and cache policy of a launch. With one or two block-rows of
// tiles (M <= 512) each B panel is read by at most two tiles, so B streams from DRAM
// about once and the shared-memory ring (two or three stages) holds too few bytes to
// cover DRAM latency; prefetching each CTA's boxes two k-blocks ahead into L2 covers
// it. With one or two block-columns (N <= 512 at 256-wide tiles) A is the streamed
// operand, so the cache roles swap too (A evict_first, B evict_last). Measured on B200
// (bench.py --mode power, sustained, cuBLASLt interleaved): 256x16384x8192 e4m3 1906 vs
// 1728 TFLOPS (cuBLASLt 1820), f16 908 vs 902 (928); 16384x256x8192 e4m3 1950 vs 1730
// (1903), f16 908 vs 907 (951). Launch-time sweeps: 512x8192x8192 f16 1232 vs 1148,
// 8192x512x8192 f16 1234 vs 1188, 256x32768x4096 (work stealing, one block-row) f16 1074
// vs 1010, e4m3 1844 vs 1743; one block-column under work stealing, sustained:
// 32768x256x4096 e4m3 1844 vs 1658 (cuBLASLt 1844), f16 894 vs 883 (947);
// 32768x128x4096 e4m3 1252 vs 1064 (1208), f16 599 vs 566 (639). Shapes with more
// block-rows and -columns, whose operands
// are re-read from L2, lose with it (8192^3 f16 1277 vs 1505), so it stays off there.
struct CachePlan {
  uint32_t policy, prefetch_k;
};
constexpr uint32_t kPrefetchK = 2;
constexpr uint32_t kL2PolicyStreamA = 4u | 8u | 16u;  // C first, A first, B last
CachePlan cache_plan(int variant, int tn, uint32_t m_tiles, uint32_t n_tiles, int sms) {
  CachePlan c{kL2Policy, 0u};
  const bool one_wave = uint64_t(m_tiles) * n_tiles <= uint64_t(sms / 2);
  if (variant == B200_VARIANT_2CTA && one_wave) {
    if (m_tiles <= 2) {
      c.prefetch_k = kPrefetchK;
    } else if (n_tiles <= 2) {
      c.prefetch_k = kPrefetchK;
      c.policy = kL2PolicyStreamA;
    }
  } else if (variant == B200_VARIANT_2CTA_CLC && m_tiles == 1) {
    c.prefetch_k = kPrefetchK;
  } else if (variant == B200_VARIANT_2CTA_CLC && n_tiles == 1 && tn <= 256) {
    c.prefetch_k = kPrefetchK;
    c.policy = kL2PolicyStreamA;
  }
  return c;
}

// C columns per tile for a pair variant when the caller leaves tile_n = 0. Chosen from
// launch-time sweeps on B200 (bench.py --mode sweep; medians of 30 launches):
//   512: the 256x512 tile cuts operand traffic by a quarter (less energy per GEMM, so a
//        higher clock under the power cap); its accumulator is single-buffered, which
//        the main loop hides from K = 1024 on, and it needs at least one full wave of
//        wide tiles: 4096^3 f16 1366 vs 1310 TFLOPS (256-wide), 8192^3 f16 711 vs 729 us
//        per launch; 8192^2 x 1024 sustained e4m3 1979 vs 1900, f16 1150 vs 1092;
//        2048x2048x8192 (32 wide tiles) 795 vs 1234.
//   128: the 256x128 tile moves 1.5x the operand bytes per flop out of L2, which caps
//        its per-pair rate (4096x1024x8192 f16: 883 vs 1279 TFLOPS for 256-wide, e4m3
//        1745 vs 2205), so it is taken only where 256-wide tiles would leave more than
//        half of the pairs idle: 2048x1024x4096 f16 686 vs 589, e4m3 911 vs 819;
//        2048x1024x8192 f16 870 vs 719, e4m3 1370 vs 1174. This is the reference's open
//        BN=64/128 choice (docs/notes/08_persistent.md:213) decided by wave count.
//   stream-K: 128 (its splits then cover twice the pairs per tile column): 1024x1024x
//        16384 f16 722 vs 690 TFLOPS (256-wide), e4m3 1177 vs 872; 512x1024x8192 f16
//        317 vs 180.
//   An explicit ring depth (`stages`) moves the choice to the next wider tile whose ring
//   holds it: the 256x128 pair stage is the largest (four atoms, two stages).
int pick_tile_n(const B200GemmArgs* a, int variant, int sms) {
  if (variant != B200_VARIANT_2CTA && variant != B200_VARIANT_2CTA_CLC &&
      variant != B200_VARIANT_2CTA_STREAMK)
    return 256;
  const int64_t pairs = sms / 2;
  // A wider tile only where it pads N no more than the next narrower one: a 512-wide
  // tile on N = 256 runs every MMA half on padding (32768x256x4096 f16 654 TFLOPS
  // against cuBLASLt's 946 before this rule), and so does a 256-wide one on N <= 128.
  const bool wide_ok = ceil_div(a->N, 512) * 2 == ceil_div(a->N, 256);
  const bool narrow_only = a->N <= 128;
  int tn = 256;
  if (variant == B200_VARIANT_2CTA_STREAMK) tn = 128;
  else if (narrow_only) tn = 128;
  else if (wide_ok && a->K >= 1024 && ceil_div(a->M, 256) * ceil_div(a->N, 512) >= pairs) tn = 512;
  else if (ceil_div(a->M, 256) * ceil_div(a->N, 256) * 2 <= pairs) tn = 128;
  if (a->stages > 0) {
    const int widest = (variant == B200_VARIANT_2CTA_STREAMK) ? 256 : 512;
    for (; tn < widest; tn *= 2) {
      VariantShape vs;
      if (variant_shape(variant, tn, &vs) == B200_OK && uint32_t(a->stages) <= vs.max_stages) break;
    }
  }
  return tn;
}

int pick_variant(const B200GemmArgs* a, int sms, bool allow_workspace) {
  const int64_t pairs = sms / 2;
  const int64_t pair_tiles = ceil_div(a->M, 256) * ceil_div(a->N, 256);
  const int64_t cta_tiles = ceil_div(a->M, 128) * ceil_div(a->N, 256);
  // A pair computes the same 256 x 256 area per SM-pair-step as two 1-CTA tiles while
  // reading each B row once per pair, so it wins whenever it needs no more waves than
  // the 1-CTA tiling (it needs more only when M rounds up badly, e.g. M = 384).
  const int64_t pair_waves = ceil_div(pair_tiles, pairs);
  const int64_t cta_waves = ceil_div(cta_tiles, sms);
  if (a->M >= 256 && pair_waves <= cta_waves) {
    // Stream-K only when 256-wide pair tiles would leave three quarters of the pairs
    // idle and K is long (>= 6144): each split tile costs an fp32 partial written and
    // read back through L2 per CTA, a few microseconds that only a long K loop repays
    // (measured, 128-wide stream-K: 1024x1024x8192 f16 518 TFLOPS vs 396 for the best
    // static tiling, e4m3 687 vs 636; 512x1024x8192 f16 317 vs 229, e4m3 373 vs 343).
    if (allow_workspace && pair_tiles * 4 <= pairs && a->K >= 6144) return B200_VARIANT_2CTA_STREAMK;
    // More than one wave (at the width pick_tile_n will choose): the persistent pairs
    // take their next tiles from cluster-launch-control work stealing (even with the
    // static order's speed: 8192^3 sustained f16 1302 vs 1293 TFLOPS, e4m3 2597 vs
    // 2580, and it adapts to SMs that run slower or are shared). One wave needs no
    // scheduler at all.
    const int tn = pick_tile_n(a, B200_VARIANT_2CTA, sms);
    const int64_t tiles = ceil_div(a->M, 256) * ceil_div(a->N, tn);
    if (tiles > pairs) return B200_VARIANT_2CTA_CLC;
    return B200_VARIANT_2CTA;
  }
  return cta_tiles > sms ? B200_VARIANT_PERSISTENT : B200_VARIANT_1CTA;
}

}  // namespace

namespace b200 {

// Everything of a launch but the launch itself: `a` is validated and non-empty,
// `sms` / `cc_major` describe the current device, and `status` is the device word
// the kernel's bounded waits report into. Shared by the C-ABI entry points and the
// plan objects (which keep the result and only launch).
int gemm_prepare(const B200GemmArgs& a, int sms, int cc_major, uint32_t* status, bool allow_workspace,
                 const GatherSpec* gather, Prepared* out) {
  int rc = B200_OK;
  if (cc_major != 10) return B200_ERR_UNSUPPORTED;
  const int ec = elem_bytes(a.c_dtype);
  std::memset(out, 0, sizeof(*out));
  if (cudaGetDevice(&out->dev) != cudaSuccess || out->dev < 0 || out->dev >= 64) return B200_ERR_CUDA;

  if (a.K == 0) {  // empty reduction: C = 0
    out->memset_only = true;
    out->c = a.C;
    out->c_pitch = size_t(a.ldc) * ec;
    out->c_width = size_t(a.N) * ec;
    out->c_height = size_t(a.M);
    return B200_OK;
  }

  const int variant = (a.variant == B200_VARIANT_AUTO) ? pick_variant(&a, sms, allow_workspace) : a.variant;
  if (variant == B200_VARIANT_2CTA_STREAMK && !allow_workspace) return B200_ERR_SCRATCH_LIMIT;
  VariantShape vs;
  const int tile_n = a.tile_n ? a.tile_n : pick_tile_n(&a, variant, sms);
  rc = variant_shape(variant, tile_n, &vs);
  if (rc != B200_OK) return rc;
  const uint32_t stages = a.stages ? uint32_t(a.stages) : vs.default_stages;
  if (stages < 2 || stages > vs.max_stages) return B200_ERR_INVALID_ARG;

  // K per TMA box (one 128-byte atom) and per pipeline stage (atoms x box)
  const uint32_t bk = (a.ab_dtype == B200_DT_E4M3) ? 128u : 64u;
  const uint32_t stage_k = bk * vs.atoms;
  const uint32_t cd_cols = 128u / uint32_t(ec);

  CUtensorMap& tA = out->tA;
  CUtensorMap& tB = out->tB;
  CUtensorMap& tC = out->tC;
  rc = encode_2d(&tA, a.A, a.ab_dtype, uint64_t(a.M), uint64_t(a.K), uint64_t(a.lda), 128u, bk);
  if (rc != B200_OK) return rc;
  // B box: the rows of one MMA's N that this CTA loads (a pair splits them)
  const uint32_t mma_n = vs.tile_n > 256u ? 256u : vs.tile_n;
  rc = encode_2d(&tB, a.B, a.ab_dtype, uint64_t(a.N), uint64_t(a.K), uint64_t(a.ldb),
                 mma_n / uint32_t(vs.cg), bk);
  if (rc != B200_OK) return rc;
  rc = encode_2d(&tC, a.C, a.c_dtype, uint64_t(a.M), uint64_t(a.N), uint64_t(a.ldc), 32u, cd_cols);
  if (rc != B200_OK) return rc;

  KParams& kp = out->kp;
  kp.M = uint32_t(a.M);
  kp.N = uint32_t(a.N);
  kp.K = uint32_t(a.K);
  kp.m_tiles = uint32_t((a.M + vs.tile_m - 1) / vs.tile_m);
  kp.n_tiles = uint32_t((a.N + vs.tile_n - 1) / vs.tile_n);
  const uint64_t tiles = uint64_t(kp.m_tiles) * kp.n_tiles;
  if (tiles > 0x7fffffffull / 4) return B200_ERR_SHAPE;
  kp.num_tiles = uint32_t(tiles);
  kp.k_blocks = uint32_t((a.K + stage_k - 1) / stage_k);
  kp.stages = stages;
  kp.group_m = a.group_m ? uint32_t(a.group_m) : uint32_t(vs.tn == 512 ? kDefaultGroupMWide : kDefaultGroupM);
  kp.fault_inject = a.fault_inject ? 1u : 0u;
  kp.scale_a = a.scale_a;
  kp.scale_b = a.scale_b;
  kp.status = status;
  kp.wait_ns = a.wait_limit_ns ? a.wait_limit_ns : kDefaultWaitNs;
  const CachePlan cp = cache_plan(variant, vs.tn, kp.m_tiles, kp.n_tiles, sms);
  kp.l2_policy = l2_policy_bits(cp.policy);
  kp.prefetch_k = prefetch_k_blocks(cp.prefetch_k);
  if (gather) {
    kp.gather = static_cast<const uint8_t*>(gather->dst);
    kp.gather_mode = gather->mode;
    kp.gather_peers = gather->peers;
    kp.gather_ld = gather->ld;
    kp.gather_col = gather->col;
  }

  const uint32_t n_sms = uint32_t(sms);
  uint32_t grid = 0;
  switch (variant) {
    case B200_VARIANT_1CTA:
    case B200_VARIANT_CLC: grid = kp.num_tiles; break;
    case B200_VARIANT_PERSISTENT: grid = kp.num_tiles < n_sms ? kp.num_tiles : n_sms; break;
    case B200_VARIANT_2CTA: {
      const uint32_t pairs = n_sms / 2;
      grid = 2u * (kp.num_tiles < pairs ? kp.num_tiles : pairs);
      break;
    }
    case B200_VARIANT_2CTA_CLC: grid = 2u * kp.num_tiles; break;
    case B200_VARIANT_2CTA_STREAMK: {
      // every pair must be resident at once (a split tile's last owner waits for
      // the partial sums of the earlier owners), so at most one pair per SM pair
      const uint64_t iters = uint64_t(kp.num_tiles) * kp.k_blocks;
      const uint32_t pairs = n_sms / 2;
      const uint32_t workers = uint32_t(iters < pairs ? iters : pairs);
      grid = 2u * workers;
      rc = streamk_workspace(out->dev, &kp.sk_work, &kp.sk_flags);
      if (rc != B200_OK) return rc;
      out->streamk = true;  // a fresh epoch is taken at every launch
      break;
    }
    default: return B200_ERR_INVALID_ARG;
  }

  out->grid = grid;
  // smem_bytes() depends only on the stage size, identical for every dtype.
  out->smem = variant_smem(vs, stages);
  out->ab = a.ab_dtype;
  out->cd = a.c_dtype;
  out->cg = vs.cg;
  out->sched = vs.sched;
  out->tn = vs.tn;
  return B200_OK;
}

// Launch a prepared GEMM on `stream` (the current device must be the one it was
// prepared on).
int gemm_launch_prepared(Prepared& pr, cudaStream_t stream) {
  if (pr.memset_only) {
    cudaError_t e = cudaMemset2DAsync(pr.c, pr.c_pitch, 0, pr.c_width, pr.c_height, stream);
    return e == cudaSuccess ? B200_OK : B200_ERR_CUDA;
  }
  LaunchPlan lp;
  lp.a = &pr.tA;
  lp.b = &pr.tB;
  lp.c = &pr.tC;
  lp.kp = pr.kp;
  lp.grid = pr.grid;
  lp.stream = stream;
  lp.smem = pr.smem;
  auto launch = [&]() -> cudaError_t {
    switch (pr.ab) {
      case B200_DT_F16: return b200::launch_f16(pr.cd, pr.cg, pr.sched, pr.tn, lp);
      case B200_DT_BF16: return b200::launch_bf16(pr.cd, pr.cg, pr.sched, pr.tn, lp);
      default: return b200::launch_e4m3(pr.cd, pr.cg, pr.sched, pr.tn, lp);
    }
  };

  cudaError_t e;
  if (pr.streamk) {
    // One workspace per device: order this launch after the previous stream-K launch
    // when that one went to another stream (inside a stream capture the caller's
    // graph edges order the launches, and nothing is recorded).
    std::lock_guard<std::mutex> lk(g_sk_mu);
    const int dev = pr.dev;
    uint32_t ep = g_sk_epoch[dev].fetch_add(1) + 1;
    if (ep == 0) ep = g_sk_epoch[dev].fetch_add(1) + 1;  // 0 is the flags' initial value
    lp.kp.sk_epoch = ep;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) return B200_ERR_CUDA;
    const bool capturing = cs != cudaStreamCaptureStatusNone;
    if (!capturing && g_sk_recorded[dev] && g_sk_last_stream[dev] != stream) {
      if (cudaStreamWaitEvent(stream, g_sk_event[dev], 0) != cudaSuccess) return B200_ERR_CUDA;
    }
    e = launch();
    if (e == cudaSuccess && !capturing) {
      if (cudaEventRecord(g_sk_event[dev], stream) != cudaSuccess) return B200_ERR_CUDA;
      g_sk_recorded[dev] = true;
      g_sk_last_stream[dev] = stream;
    }
  } else {
    e = launch();
  }
  if (e == cudaErrorNotSupported) return B200_ERR_UNSUPPORTED;
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return B200_ERR_LAUNCH;
  }
  return B200_OK;
}

int gemm_launch_impl(const B200GemmArgs& a, cudaStream_t stream, int sms, int cc_major,
                     uint32_t* status, bool allow_workspace, const GatherSpec* gather) {
  Prepared pr;
  int rc = gemm_prepare(a, sms, cc_major, status, allow_workspace, gather, &pr);
  if (rc != B200_OK) return rc;
  return gemm_launch_prepared(pr, stream);
}

}  // namespace b200

extern "C" {

int b200_gemm_abi_version(void) { return B200GEMM_ABI_VERSION; }

const char* b200_gemm_strerror(int code) {
  switch (code) {
    case B200_OK: return "ok";
    case B200_ERR_INVALID_ARG: return "invalid argument (null pointer, dtype or variant)";
    case B200_ERR_SHAPE: return "invalid shape or leading dimension";
    case B200_ERR_ALIGN: return "pointer or row stride is not 16-byte aligned";
    case B200_ERR_TMAP: return "tensor-map encoding failed";
    case B200_ERR_LAUNCH: return "kernel launch failed";
    case B200_ERR_DEVICE_TIMEOUT: return "a bounded device wait timed out";
    case B200_ERR_UNSUPPORTED: return "unsupported dtype/variant or device (needs sm_100)";
    case B200_ERR_CUDA: return "CUDA runtime error";
    case B200_ERR_SCRATCH_LIMIT:
      return "request needs more scratch than the allocation-free entry point's static array holds";
    default: return "unknown error code";
  }
}

int b200_gemm_variant_info(int32_t variant, int32_t ab_dtype, int32_t* tile_m, int32_t* tile_n,
                           int32_t* max_stages, int32_t* default_stages) {
  if (ab_dtype != B200_DT_F16 && ab_dtype != B200_DT_BF16 && ab_dtype != B200_DT_E4M3)
    return B200_ERR_INVALID_ARG;
  VariantShape vs;
  int rc = variant_shape(variant, tile_n ? *tile_n : 0, &vs);
  if (rc != B200_OK) return rc;
  if (tile_m) *tile_m = static_cast<int32_t>(vs.tile_m);
  if (tile_n) *tile_n = static_cast<int32_t>(vs.tile_n);
  if (max_stages) *max_stages = static_cast<int32_t>(vs.max_stages);
  if (default_stages) *default_stages = static_cast<int32_t>(vs.default_stages);
  return B200_OK;
}

// Argument checks that need no GPU (shared by b200_gemm and b200_gemm_pick_variant).
static int validate(const B200GemmArgs* a) {
  if (!a) return B200_ERR_INVALID_ARG;
  if (a->ab_dtype != B200_DT_F16 && a->ab_dtype != B200_DT_BF16 && a->ab_dtype != B200_DT_E4M3)
    return B200_ERR_INVALID_ARG;
  if (a->c_dtype != B200_DT_F16 && a->c_dtype != B200_DT_BF16 && a->c_dtype != B200_DT_F32)
    return B200_ERR_INVALID_ARG;
  if (a->variant < B200_VARIANT_AUTO || a->variant > B200_VARIANT_2CTA_STREAMK) return B200_ERR_INVALID_ARG;
  if (a->M < 0 || a->N < 0 || a->K < 0) return B200_ERR_SHAPE;
  // TMA coordinates are int32 and the tile counters are uint32.
  const int64_t lim = (int64_t(1) << 31) - 1;
  if (a->M > lim || a->N > lim || a->K > lim) return B200_ERR_SHAPE;
  if (a->group_m < 0 || a->stages < 0 || a->reserved != 0) return B200_ERR_INVALID_ARG;
  if (a->tile_n != 0 && a->tile_n != 128 && a->tile_n != 256 && a->tile_n != 512) return B200_ERR_INVALID_ARG;
  if (a->M == 0 || a->N == 0) return B200_OK;
  if (a->ldc < a->N) return B200_ERR_SHAPE;
  if (!a->C) return B200_ERR_INVALID_ARG;
  const int eb = elem_bytes(a->ab_dtype), ec = elem_bytes(a->c_dtype);
  if (!aligned16(a->C) || (a->ldc * ec) % 16) return B200_ERR_ALIGN;
  if (a->K == 0) return B200_OK;  // A and B are not read: C = 0
  if (a->lda < a->K || a->ldb < a->K) return B200_ERR_SHAPE;
  if (!a->A || !a->B) return B200_ERR_INVALID_ARG;
  if (!aligned16(a->A) || !aligned16(a->B)) return B200_ERR_ALIGN;
  if ((a->lda * eb) % 16 || (a->ldb * eb) % 16) return B200_ERR_ALIGN;
  // TMA global strides must stay below 2^40 bytes.
  if (a->lda * eb >= (int64_t(1) << 40) || a->ldb * eb >= (int64_t(1) << 40) ||
      a->ldc * ec >= (int64_t(1) << 40))
    return B200_ERR_SHAPE;
  if ((a->scale_a && (reinterpret_cast<uintptr_t>(a->scale_a) & 3u)) ||
      (a->scale_b && (reinterpret_cast<uintptr_t>(a->scale_b) & 3u)))
    return B200_ERR_ALIGN;
  return B200_OK;
}

int b200_gemm_pick_variant(const B200GemmArgs* args) {
  int rc = validate(args);
  if (rc != B200_OK) return rc;
  if (args->variant != B200_VARIANT_AUTO) return args->variant;
  int dev = 0;
  rc = device_setup(&dev);
  if (rc != B200_OK) return rc;
  return pick_variant(args, g_sm_count[dev], true);
}

int b200_gemm_pick_config(const B200GemmArgs* args, int32_t* variant, int32_t* tile_n) {
  int rc = validate(args);
  if (rc != B200_OK) return rc;
  if (!variant || !tile_n) return B200_ERR_INVALID_ARG;
  int dev = 0;
  rc = device_setup(&dev);
  if (rc != B200_OK) return rc;
  const int v = args->variant == B200_VARIANT_AUTO ? pick_variant(args, g_sm_count[dev], true) : args->variant;
  *variant = v;
  *tile_n = args->tile_n ? args->tile_n : pick_tile_n(args, v, g_sm_count[dev]);
  return B200_OK;
}

int b200_gemm(const B200GemmArgs* args, void* stream_v) {
  int rc = validate(args);
  if (rc != B200_OK) return rc;
  const B200GemmArgs& a = *args;
  if (a.M == 0 || a.N == 0) return B200_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  int dev = 0;
  rc = device_setup(&dev);
  if (rc != B200_OK) return rc;
  return b200::gemm_launch_impl(a, stream, g_sm_count[dev], g_cc_major[dev], status_word(dev));
}

struct B200GemmPlan {
  bool empty;  // M == 0 or N == 0: launching does nothing
  b200::Prepared pr;
};

int b200_gemm_plan_create(const B200GemmArgs* args, B200GemmPlan** plan) {
  if (!plan) return B200_ERR_INVALID_ARG;
  *plan = nullptr;
  int rc = validate(args);
  if (rc != B200_OK) return rc;
  int dev = 0;
  rc = device_setup(&dev);
  if (rc != B200_OK) return rc;
  B200GemmPlan* p = new (std::nothrow) B200GemmPlan();
  if (!p) return B200_ERR_CUDA;
  p->empty = args->M == 0 || args->N == 0;
  if (!p->empty) {
    rc = b200::gemm_prepare(*args, g_sm_count[dev], g_cc_major[dev], status_word(dev), true, nullptr, &p->pr);
    if (rc != B200_OK) {
      delete p;
      return rc;
    }
  }
  *plan = p;
  return B200_OK;
}

int b200_gemm_plan_launch(B200GemmPlan* plan, void* stream_v) {
  if (!plan) return B200_ERR_INVALID_ARG;
  if (plan->empty) return B200_OK;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return B200_ERR_CUDA;
  if (dev != plan->pr.dev) return B200_ERR_INVALID_ARG;
  return b200::gemm_launch_prepared(plan->pr, static_cast<cudaStream_t>(stream_v));
}

void b200_gemm_plan_destroy(B200GemmPlan* plan) { delete plan; }

int b200_gemm_allgather(const B200GemmArgs* args, const void* dst, int32_t mode, int32_t npeers,
                        int64_t ldg, int64_t col_off, void* stream_v) {
  int rc = validate(args);
  if (rc != B200_OK) return rc;
  const B200GemmArgs& a = *args;
  if (!dst || (mode != B200_GATHER_MULTICAST && mode != B200_GATHER_PEERS)) return B200_ERR_INVALID_ARG;
  if (mode == B200_GATHER_PEERS && (npeers < 1 || npeers > 64)) return B200_ERR_INVALID_ARG;
  if (a.M == 0 || a.N == 0) return B200_OK;
  if (a.K == 0) return B200_ERR_SHAPE;  // the gathered copy is written by the GEMM epilogue
  const int64_t ec = elem_bytes(a.c_dtype);
  if (ldg < 0 || col_off < 0 || ldg < col_off + a.N) return B200_ERR_SHAPE;
  if ((a.N * ec) % 16 || (ldg * ec) % 16 || (col_off * ec) % 16 || !aligned16(dst)) return B200_ERR_ALIGN;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  int dev = 0;
  rc = device_setup(&dev);
  if (rc != B200_OK) return rc;
  // Every schedule but stream-K (whose partial-tile workspace this entry point does
  // not take): AUTO resolves as for b200_gemm without the workspace.
  if (a.variant == B200_VARIANT_2CTA_STREAMK) return B200_ERR_UNSUPPORTED;
  const B200GemmArgs& a2 = a;
  b200::GatherSpec g{dst, uint32_t(mode), uint32_t(mode == B200_GATHER_PEERS ? npeers : 0), uint64_t(ldg),
                     uint64_t(col_off)};
  return b200::gemm_launch_impl(a2, stream, g_sm_count[dev], g_cc_major[dev], status_word(dev), false, &g);
}

int b200_gemm_status(void* stream_v, int clear, uint32_t* bits) {
  int dev = 0;
  int rc = device_setup(&dev);
  if (rc != B200_OK) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (cudaStreamSynchronize(stream) != cudaSuccess) return B200_ERR_CUDA;
  uint32_t v = 0;
  if (cudaMemcpy(&v, status_word(dev), sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess)
    return B200_ERR_CUDA;
  if (clear && v) {
    if (cudaMemset(status_word(dev), 0, sizeof(uint32_t)) != cudaSuccess) return B200_ERR_CUDA;
  }
  if (bits) *bits = v;
  return v ? B200_ERR_DEVICE_TIMEOUT : B200_OK;
}

}  // extern "C"

namespace b200 {

int gemm_validate(const B200GemmArgs* a) { return validate(a); }

int gemm_resolve_driver() {
  std::lock_guard<std::mutex> lk(g_mu);
  return resolve_encode();
}

}  // namespace b200
