/* b200gemm.h — C ABI of the B200 (sm_100a) dense GEMM library, libb200gemm.so.
 *
 * The reference (TheManWhoIsStupid/Hopper-lab) has no library and no FFI: each
 * experiment carries its kernel launcher in an anonymous namespace,
 *   launch_config<S,...>(tmap_a, tmap_b, tmap_d, D, M, N, K[, group_m])   and
 *   dispatch(stages, flag, ...)
 * (src/05_gemm/gemm_ws.cu:201-235, src/07_fp8/gemm_fp8.cu:188-215,
 *  src/08_persistent/gemm_fp8_persist.cu:222-270, src/08_persistent/gemm_fp8_bn128.cu:256-311).
 * b200_gemm() replaces all of those launchers with one entry point: it encodes the
 * tensor maps itself (the reference's make_tmap_h / make_tmap_fp8 / make_tmap_f,
 * src/05_gemm/gemm_ws.cu:162-199), validates shape and alignment, and launches on
 * the caller's stream.
 *
 * Conventions
 *   - Layout "TN": A is M x K row-major, B is N x K row-major (K contiguous), C is
 *     M x N row-major; C = scale_a * scale_b * A . B^T with fp32 accumulation.
 *   - All pointers are device pointers of the current CUDA device.
 *   - Never exits the process (the reference's launchers exit on error,
 *     include/common/errors.h:8-16); every failure is a negative return code.
 *   - Stream-ordered and asynchronous; thread-safe; no allocation on the hot path
 *     (the per-device status word is allocated once, on the first call on a device;
 *     the stream-K workspace, 32 MB, once on the first stream-K call on a device).
 *   - Stream-K launches on one device share that workspace, so the library orders
 *     them: a stream-K launch on a stream other than the previous stream-K launch's
 *     first waits (cudaStreamWaitEvent) for that launch to finish. Inside a stream
 *     capture nothing is recorded or waited for; the captured graph must order its
 *     stream-K launches itself (one stream, or explicit dependencies).
 *   - Device-side waits are bounded: a protocol failure sets the device status
 *     word, which b200_gemm_status() reads back as B200_ERR_DEVICE_TIMEOUT.
 */
#ifndef B200GEMM_H_
#define B200GEMM_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200GEMM_ABI_VERSION 4

/* element types */
enum {
  B200_DT_F16 = 0,  /* IEEE binary16                              */
  B200_DT_BF16 = 1, /* bfloat16                                   */
  B200_DT_E4M3 = 2, /* fp8 e4m3 (OCP "fn": no inf, max 448)       */
  B200_DT_F32 = 3   /* output only                                */
};

/* kernel variants (the reference experiment each one succeeds) */
enum {
  B200_VARIANT_AUTO = 0,       /* library picks                                        */
  B200_VARIANT_1CTA = 1,       /* one 128x256 tile per CTA    (05_gemm gemm_ws)        */
  B200_VARIANT_2CTA = 2,       /* cta_group::2 pair, 256x256 or 256x512 tile,
                                  persistent static schedule (06_cluster gemm_ws_cluster)*/
  B200_VARIANT_PERSISTENT = 3, /* 1-CTA, grid = SM count, static group-M schedule
                                                              (08_persistent persist)  */
  B200_VARIANT_CLC = 4,        /* 1-CTA, cluster-launch-control work stealing
                                                              (08_persistent bn128 dyn)*/
  B200_VARIANT_2CTA_CLC = 5,   /* cta_group::2 pair + cluster-launch-control work
                                  stealing (the pair form of the persistent kernel) */
  B200_VARIANT_2CTA_STREAMK = 6 /* cta_group::2 pair, stream-K: every pair takes an equal
                                  share of the tile x k-block iterations; split tiles are
                                  summed in a fixed order through a library-owned fp32
                                  workspace; AUTO takes it only when 256-wide tiles
                                  would leave three quarters of the pairs idle and K is
                                  at least 6144                                          */
};

/* return codes */
enum {
  B200_OK = 0,
  B200_ERR_INVALID_ARG = -1,   /* null args / pointers, unknown dtype or variant      */
  B200_ERR_SHAPE = -2,         /* negative or oversize dims, ld < K or ld < N          */
  B200_ERR_ALIGN = -3,         /* pointer or row stride not 16-byte aligned            */
  B200_ERR_TMAP = -4,          /* cuTensorMapEncodeTiled rejected a descriptor         */
  B200_ERR_LAUNCH = -5,        /* CUDA launch / attribute error                        */
  B200_ERR_DEVICE_TIMEOUT = -6,/* a bounded device wait gave up (see b200_gemm_status) */
  B200_ERR_UNSUPPORTED = -7,   /* dtype/variant combination not built, or not sm_100   */
  B200_ERR_CUDA = -8,          /* other CUDA runtime error                             */
  B200_ERR_SCRATCH_LIMIT = -9  /* b200_gemm_noalloc: request needs more scratch than its
                                  static device array holds                             */
};

typedef struct B200GemmArgs {
  int32_t ab_dtype;        /* B200_DT_F16 | B200_DT_BF16 | B200_DT_E4M3 (A and B)        */
  int32_t c_dtype;         /* B200_DT_F16 | B200_DT_BF16 | B200_DT_F32                   */
  int64_t M, N, K;
  int64_t lda, ldb, ldc;   /* elements; lda >= K, ldb >= K, ldc >= N                     */
  const void* A;           /* M x lda                                                    */
  const void* B;           /* N x ldb                                                    */
  void* C;                 /* M x ldc                                                    */
  const float* scale_a;    /* device fp32 scalar or NULL (1.0)                           */
  const float* scale_b;    /* device fp32 scalar or NULL (1.0)                           */
  int32_t variant;         /* B200_VARIANT_*                                             */
  int32_t group_m;         /* group-M swizzle width, 0 = library default                 */
  int32_t stages;          /* smem ring depth, 0 = library default                       */
  int32_t fault_inject;    /* 0 in production; 1 = test hook: producer issues no loads,
                              so the bounded waits must report a device timeout          */
  uint64_t wait_limit_ns;  /* bound of each device wait, 0 = library default (1 s)       */
  int32_t tile_n;          /* C columns per tile: 0 = library default, 128, 256 or 512.
                              1-CTA variants: 256 only; pair variants: 128, 256, 512
                              (stream-K: 128 or 256). The default picks by wave count:
                              512 for K >= 1024 with a full wave of wide tiles, 128
                              where 256-wide tiles would leave pairs idle or N <= 128,
                              else 256; never a width that pads N more than the next
                              narrower one;
                              with `stages` given, the next wider tile whose ring
                              holds that many stages                                    */
  int32_t reserved;        /* must be 0                                                  */
} B200GemmArgs;

/* Launch C = scale_a*scale_b*A.B^T on `stream` (a cudaStream_t, NULL = legacy default). */
int b200_gemm(const B200GemmArgs* args, void* stream);

/* Human-readable text of a return code. */
const char* b200_gemm_strerror(int code);

/* Synchronise `stream`, then read (and clear when `clear` != 0) the device status
 * word of the current device. Returns B200_OK, B200_ERR_DEVICE_TIMEOUT (and stores
 * the raw bits in *bits when bits != NULL) or B200_ERR_CUDA. */
int b200_gemm_status(void* stream, int clear, uint32_t* bits);

/* Library facts: tile shape and stage limits of a variant at a tile width
 * (`tile_n` in: 0 = the variant's default width; out: the width used), for hosts
 * and tests. Returns B200_OK or B200_ERR_INVALID_ARG. */
int b200_gemm_variant_info(int32_t variant, int32_t ab_dtype, int32_t* tile_m, int32_t* tile_n,
                           int32_t* max_stages, int32_t* default_stages);

/* The variant B200_VARIANT_AUTO resolves to for this problem on the current device. */
int b200_gemm_pick_variant(const B200GemmArgs* args);

/* The variant and tile width b200_gemm would launch for `args` on the current device
 * (AUTO and tile_n = 0 resolved; explicit choices returned as given). Returns B200_OK
 * or the code b200_gemm's argument checks would return. The reference fixes both per
 * experiment at compile time (src/08_persistent/gemm_fp8_bn128.cu:73 is its BN=128
 * kernel); this call exposes the library's choice to hosts, benches and tests. */
int b200_gemm_pick_config(const B200GemmArgs* args, int32_t* variant, int32_t* tile_n);

/* Allocation-free form of b200_gemm, for callers that cannot have a library call
 * cudaMalloc: code inside frameworks whose pool allocator must own every device
 * allocation, processes whose device footprint is fixed after start-up, and paths
 * that must not take the allocator's locks. Same arguments, kernels and results as
 * b200_gemm. The kernel's scratch (its status word) lives in a 256-byte static
 * device array that every GPU loading the library holds until exit; a request
 * needing more scratch returns B200_ERR_SCRATCH_LIMIT (the GEMM needs 4 bytes for
 * every shape). All calls share that array and each call clears its word first,
 * so calls that overlap on the GPU race on the status. The first call on a device
 * looks up the array's device address (do it before any stream capture). With
 * check_status != 0 the call synchronises `stream` and returns
 * B200_ERR_DEVICE_TIMEOUT if a bounded wait gave up. No counterpart in the
 * reference. */
int b200_gemm_noalloc(const B200GemmArgs* args, void* stream, int check_status);

/* Plans: everything b200_gemm resolves per call (argument checks, variant and tile
 * choice, the three tensor maps, kernel parameters, grid) done once, for callers that
 * launch the same GEMM on the same buffers repeatedly (serving loops, benchmark
 * steps). A plan is bound to the pointers in `args` and to the current device at
 * creation; b200_gemm_plan_launch only launches (B200_ERR_INVALID_ARG on another
 * device). The reference encodes its tensor maps once per experiment and passes them
 * to dispatch() (src/05_gemm/gemm_ws.cu:214-235); a plan is that split as an API.
 * Plans own host memory only; destroy them with b200_gemm_plan_destroy. */
typedef struct B200GemmPlan B200GemmPlan;
int b200_gemm_plan_create(const B200GemmArgs* args, B200GemmPlan** plan);
int b200_gemm_plan_launch(B200GemmPlan* plan, void* stream);
void b200_gemm_plan_destroy(B200GemmPlan* plan);

/* Fused GEMM + all-gather of C across the GPUs of one node. Computes this GPU's
 * C = scale_a*scale_b*A.B^T exactly as b200_gemm does (C is written locally too) and,
 * from the same epilogue, stores every finished C tile into the gathered matrix G of
 * every GPU: G[row * ldg + col_off + col] = C[row][col], element type of C. The
 * transfer runs tile by tile under the main loop of the following tiles, over NVLink:
 *   B200_GATHER_MULTICAST  `dst` is the multicast (NVLS) address of a buffer bound on
 *                          every GPU; one multimem.st per 16 bytes reaches all of them
 *                          through the NVSwitch.
 *   B200_GATHER_PEERS      `dst` is a device array of `npeers` uint64 base addresses of
 *                          peer-mapped buffers (this GPU's own included); each tile is
 *                          stored to every one of them.
 * Requirements (else B200_ERR_ALIGN / B200_ERR_SHAPE / B200_ERR_INVALID_ARG): K > 0;
 * N, ldg and col_off keep 16-byte chunks of C whole and aligned (N * elem, ldg * elem
 * and col_off * elem multiples of 16); ldg >= col_off + N; dst 16-byte aligned (and
 * every base in the array). On return the launch is queued; G is complete on a GPU
 * once every GPU's launch has completed, so the caller synchronises the GPUs (e.g. a
 * barrier on the symmetric-memory signal pads) before reading G. Every schedule but
 * stream-K (whose workspace this entry point does not take; it returns
 * B200_ERR_UNSUPPORTED); AUTO resolves as b200_gemm's does without stream-K. The
 * reference has no
 * multi-GPU code; its planned counterpart is a separate ncclAllGather after the GEMM. */
enum { B200_GATHER_MULTICAST = 1, B200_GATHER_PEERS = 2 };
int b200_gemm_allgather(const B200GemmArgs* args, const void* dst, int32_t mode, int32_t npeers,
                        int64_t ldg, int64_t col_off, void* stream);

/* Per-tensor e4m3 quantiser on the device: *scale = amax(|x|)/448 (1 when all
 * x == 0) and q[i] = e4m3_rn_satfinite(x[i] / *scale). Device pointers: x (fp32,
 * 16-byte aligned), q (n bytes, 8-byte aligned), scale (one fp32). Replaces the
 * reference's host-side `quantize` (src/07_fp8/gemm_fp8.cu:182-186), which casts
 * without a scale. Stream-ordered; returns B200_OK or a negative code. */
int b200_quantize_e4m3(const float* x, int64_t n, void* q, float* scale, void* stream);

/* ABI version (B200GEMM_ABI_VERSION). */
int b200_gemm_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* B200GEMM_H_ */
