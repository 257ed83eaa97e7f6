// gemm_sm100.cuh — warp-specialised tcgen05 GEMM for B200 (sm_100a).
//
//   C[M,N] = scale_a * scale_b * (A[M,K] · B[N,K]^T),  fp32 accumulation in TMEM
//
// Layout contract ("TN"), identical to the reference's GEMM experiments
// (src/05_gemm/gemm_ws.cu:258-265, src/07_fp8/gemm_fp8.cu:246-253): A is M×K
// row-major, B is stored N×K (K contiguous), C is M×N row-major. Leading
// dimensions are free (lda ≥ K, ldb ≥ K, ldc ≥ N, 16-byte multiples).
//
// What each reference kernel becomes here:
//   gemm_ws_kernel   (src/05_gemm/gemm_ws.cu:56)   -> CG=1, one tile per CTA
//   gemm_ws_cluster  (src/06_cluster/gemm_ws_cluster.cu:50) -> CG=2: the CTA pair
//                    runs one cta_group::2 MMA (M=256) and each CTA loads half of
//                    B, so the pair shares B without any multicast load
//   gemm_fp8_kernel  (src/07_fp8/gemm_fp8.cu:48)   -> AB = e4m3, kind::f8f6f4,
//                    per-tensor fp32 scales fused in the epilogue
//   gemm_fp8_persist (src/08_persistent/gemm_fp8_persist.cu:68) -> SCHED_STATIC
//                    (grid = resident CTAs, tile += grid, group-M order)
//   gemm_fp8_bn128   (src/08_persistent/gemm_fp8_bn128.cu:73, dynamic queue, BN=128)
//                    -> SCHED_CLC: hardware cluster-launch-control work stealing
//                    replaces the global atomic tile counter; TN = 128 is the narrow
//                    tile (256 x 128 per pair) for problems whose 256-wide tiles
//                    leave pairs idle
//
// CTA = 384 threads, 12 warps:
//   warp 0      TMA producer (one lane): A/B k-blocks into an S-stage smem ring
//               (one 128-byte K atom per stage for 1-CTA and 512-wide tiles, two
//               for the other pair tiles)
//   warp 1      TMEM owner + MMA issuer (one lane of the leader CTA)
//   warp 2      CLC scheduler (one lane of the leader CTA; SCHED_CLC only)
//   warp 3      idle
//   warps 4-11  epilogue: TMEM -> registers -> (scale, narrow) -> swizzled smem ->
//               TMA store; warp 4+4e+q drains TMEM lanes 32q..32q+31, columns of half
//               e of each accumulator slot
// TN is the tile width (C columns per tile): 128, 256 or 512. One MMA is
// MMA_N = min(TN, 256) wide and TMEM holds two MMA_N-column fp32 slots. A tile of one
// MMA width (TN = 128 or 256) uses one slot, so the epilogue of tile t overlaps the
// main loop of tile t+1. A pair tile of TN = 512 (two N=256 MMAs per K-step sharing
// the A tiles, 25% less operand traffic per flop) uses both slots; the epilogue
// releases each slot as soon as it is drained, and the next tile's first MMAs into
// that slot start then.
#pragma once

#include "sm100_ptx.cuh"

namespace b200 {

enum : int { DT_F16 = 0, DT_BF16 = 1, DT_E4M3 = 2, DT_F32 = 3 };
enum : int { SCHED_STATIC = 0, SCHED_CLC = 1, SCHED_STREAMK = 2 };

// Bits OR-ed into the device status word when a bounded wait gives up.
enum : uint32_t {
  ST_PRODUCER_EMPTY = 1u << 0,
  ST_MMA_FULL = 1u << 1,
  ST_MMA_TMEM_EMPTY = 1u << 2,
  ST_EPI_TMEM_FULL = 1u << 3,
  ST_SCHED = 1u << 4,
  ST_DRAIN = 1u << 5,
  ST_STREAMK = 1u << 6,
  ST_ABORTED = 1u << 31,
};

struct KParams {
  uint32_t M, N, K;
  uint32_t m_tiles;    // ceil(M / (128*CG))
  uint32_t n_tiles;    // ceil(N / TN)
  uint32_t num_tiles;  // m_tiles * n_tiles
  uint32_t k_blocks;   // ceil(K / BK)
  uint32_t stages;     // smem ring depth (runtime, ≤ the kernel's maximum)
  uint32_t group_m;    // group-M swizzle width (≥ 1)
  uint32_t fault_inject;  // test hook: 1 = the producer issues no loads
  const float* scale_a;   // device, per-tensor, may be null (= 1)
  const float* scale_b;
  uint32_t* status;       // device status word, may be null
  uint64_t wait_ns;       // bound of every mbarrier wait
  // L2 cache policies: bit 0 A loads evict_last (A panels are reused by every wave of a
  // group-M group), bit 1 B loads evict_first (a B panel's reuse is within one wave),
  // bit 2 C stores evict_first (C is never read back); the mirrored roles, for shapes
  // whose A is the streamed operand: bit 3 A loads evict_first (when bit 0 is clear),
  // bit 4 B loads evict_last (when bit 1 is clear); 0 = evict_normal everywhere
  uint32_t l2_policy;
  // L2 prefetch distance in k-blocks (0 = off): with the loads of k-block kb the producer
  // prefetches this CTA's boxes of k-block kb + prefetch_k into L2, so that a DRAM-streamed
  // operand has more bytes in flight than the shared-memory ring holds
  uint32_t prefetch_k;
  // SCHED_STREAMK only: fp32 partial-tile workspace (one 128 x MMA_N region per CTA
  // slot), per-slot ready flags, and this launch's epoch (the value a ready flag
  // holds; flags never need resetting between launches)
  float* sk_work;
  uint32_t* sk_flags;
  uint32_t sk_epoch;
  // Fused all-gather of C (b200_gemm_allgather): every C tile is also stored at
  // gather[row * gather_ld + gather_col + col] on every GPU of the node.
  //   GATHER_MULTICAST: `gather` is a multicast (NVLS) address, one multimem.st per 16 B
  //   GATHER_PEERS    : `gather` is a device array of `gather_peers` peer-mapped bases
  const uint8_t* gather;
  uint32_t gather_mode;
  uint32_t gather_peers;
  uint64_t gather_ld;   // elements
  uint64_t gather_col;  // elements
};
enum : uint32_t { GATHER_OFF = 0, GATHER_MULTICAST = 1, GATHER_PEERS = 2 };

// A unit of work of one CTA (pair): k-blocks [kb0, kb1) of a tile.
//   FULL    the whole K range: store C
//   PARTIAL the range ends inside the tile: write fp32 partial sums, raise the flag
//   LAST    the range ends the tile but starts inside it: add the partials of the
//           workers that own the earlier part of the tile, then store C
enum : uint32_t { ITEM_FULL = 0, ITEM_PARTIAL = 1, ITEM_LAST = 2 };
struct WorkItem {
  uint32_t tile, kb0, kb1, kind, idx;
};

// Linear tile id -> (block-row, block-col) in group-M order. Same mapping as the
// reference's tile_to_bmn (src/08_persistent/gemm_fp8_persist.cu:56-66): groups of
// G block-rows, block-row fastest inside a group; G = 1 is plain row-wave order.
__host__ __device__ inline void tile_to_bmn(uint32_t tile, uint32_t num_bm, uint32_t num_bn,
                                            uint32_t G, uint32_t& bm, uint32_t& bn) {
  const uint32_t per_group = G * num_bn;
  const uint32_t g = tile / per_group;
  const uint32_t first_bm = g * G;
  const uint32_t rem = num_bm - first_bm;
  const uint32_t gsize = rem < G ? rem : G;
  const uint32_t t = tile - g * per_group;
  bm = first_bm + t % gsize;
  bn = t / gsize;
}

// K atoms per pipeline stage of the 256x256 and 256x128 pair tiles (compile-time options
// so that a second build can compare them; the stage count follows from the shared
// memory left).
#ifndef B200_PAIR_ATOMS_256
#define B200_PAIR_ATOMS_256 2
#endif
#ifndef B200_PAIR_ATOMS_128
#define B200_PAIR_ATOMS_128 4
#endif

template <int AB, int CD, int CG, int SCHED, int TN>
struct GemmCfg {
  static constexpr int BM = 128;                       // rows of C per CTA
  static constexpr int MMA_N = TN > 256 ? 256 : TN;    // N of one tcgen05.mma
  static constexpr int NH = TN / MMA_N;                // MMAs (accumulator slots) per tile
  static constexpr int BN = TN;                        // columns of C per tile
  static constexpr int KIND = (AB == DT_E4M3) ? 1 : 0; // 0 kind::f16, 1 kind::f8f6f4
  static constexpr int AB_BYTES = (AB == DT_E4M3) ? 1 : 2;
  // One 128-byte swizzle atom of K per TMA box. A pair stage of one MMA width carries
  // B200_PAIR_ATOMS_256 / _128 atoms: two for 256x256 (64 KB, three stages) and four for
  // 256x128 (96 KB, two stages). Fewer, larger stages mean fewer commit / barrier round
  // trips per MMA, and each costs tensor-pipe time; the narrow tile's MMAs are half as
  // long, so it gains from four atoms where the 256-wide tile loses with three (two
  // 96 KB stages leave too little overlap for its longer stage). 1-CTA stages and
  // 512-wide pair stages are already 48 KB and keep one atom so that four fit.
  static constexpr int ATOMS =
      (CG == 2 && NH == 1) ? (MMA_N == 128 ? B200_PAIR_ATOMS_128 : B200_PAIR_ATOMS_256) : 1;
  static constexpr int ATOM_K = 128 / AB_BYTES;        // elements of K per atom
  static constexpr int BK = ATOMS * ATOM_K;            // elements of K per stage
  static constexpr int KSTEPS = 4 * ATOMS;             // 32-byte MMA K-steps per stage
  static constexpr int B_HALF_ROWS = MMA_N / CG;       // rows of B per CTA per MMA
  static constexpr uint32_t B_HALF = B_HALF_ROWS * 128; // bytes of one MMA's B in one atom
  static constexpr uint32_t A_ATOM = BM * 128;         // bytes
  static constexpr uint32_t B_ATOM = NH * B_HALF;
  static constexpr uint32_t A_STAGE = ATOMS * A_ATOM;
  static constexpr uint32_t B_STAGE = ATOMS * B_ATOM;
  static constexpr uint32_t STAGE = A_STAGE + B_STAGE;
  static constexpr int CD_BYTES = (CD == DT_F32) ? 4 : 2;
  static constexpr int EPI_COLS = 128 / CD_BYTES;      // C columns per 128-byte chunk
  static constexpr int EPI_CHUNKS = MMA_N / EPI_COLS; // per accumulator slot
  static constexpr uint32_t EPI_BUF = 32 * 128;        // 32 rows × 128 bytes
  // Eight epilogue warps: warp 4 + 4e + q drains TMEM lane quarter q, column half e
  // of each slot, staging through one 4 KB buffer of its own.
  static constexpr int EPI_WARPS = 8;
  static constexpr int EPI_CHUNKS_PER_WARP = EPI_CHUNKS / 2;
  static constexpr int EPI_VALS = EPI_CHUNKS_PER_WARP * EPI_COLS;  // fp32 values per thread
  static constexpr uint32_t EPI_BYTES = EPI_WARPS * EPI_BUF;
  static constexpr uint32_t TMEM_COLS = 2 * MMA_N;     // two MMA_N-column fp32 slots
  static constexpr uint32_t MMA_M = BM * CG;
  static constexpr uint32_t IDESC =
      idesc_f32acc(AB == DT_BF16 ? 1u : 0u, AB == DT_BF16 ? 1u : 0u, MMA_M, MMA_N);
  static constexpr uint32_t MAX_SMEM = 232448;         // 227 KB opt-in per CTA
  static constexpr uint32_t BAR_BYTES = 448;
  // CLC response ring depth: the scheduler may run this many tiles ahead of the
  // slowest consumer (at small K a tile is only a few stages long, and a
  // try_cancel round trip plus the pair forwarding must fit in the lead).
  static constexpr uint32_t CLC_SLOTS = 4;
  static constexpr uint32_t ALIGN_SLACK = 1024;
  static constexpr uint32_t MAX_STAGES =
      (MAX_SMEM - EPI_BYTES - BAR_BYTES - ALIGN_SLACK) / STAGE;
  static constexpr uint32_t NUM_THREADS = 128 + 32 * EPI_WARPS;
  // CLC ring consumers per CTA: producer + MMA + the epilogue warps
  static constexpr uint32_t SCHED_CONSUMERS = 2 + EPI_WARPS;

  static uint32_t smem_bytes(uint32_t stages) {
    return stages * STAGE + EPI_BYTES + BAR_BYTES + ALIGN_SLACK;
  }
  static_assert(TN == 128 || TN == 256 || TN == 512, "tile widths 128, 256 and 512");
  static_assert(NH == 1 || CG == 2, "512-wide tiles are built for CTA pairs");
  static_assert(TN != 128 || CG == 2, "128-wide tiles are built for CTA pairs");
  static_assert(SCHED != SCHED_STREAMK || NH == 1, "stream-K uses tiles of one MMA width");
  static_assert(EPI_CHUNKS_PER_WARP >= 1, "every epilogue warp owns at least one chunk");
  // stream-K partial of one CTA: 128 rows x MMA_N fp32 columns
  static constexpr uint32_t SK_FLOATS = BM * MMA_N;
  static_assert(MAX_STAGES <= 8, "the barrier block holds 8 ring stages");
  static_assert(CLC_SLOTS <= 8, "the barrier block holds 8 CLC response slots");
};

template <int AB, int CD, int CG, int SCHED, int TN>
__global__ void __launch_bounds__(384, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const KParams p) {
  using Cfg = GemmCfg<AB, CD, CG, SCHED, TN>;
  constexpr int NH = Cfg::NH;
  extern __shared__ uint8_t smem_raw[];

  // ---- shared-memory carve-up (1024-byte aligned for SWIZZLE_128B) ----
  // Same offsets in both CTAs of a pair: the MMA reads the peer's operand tiles at
  // the addresses it names for its own, and commits land on the peer's barriers.
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw);
  const uint32_t S = p.stages;
  const uint32_t sA = base;
  const uint32_t sB = base + S * Cfg::A_STAGE;
  const uint32_t sEpi = base + S * Cfg::STAGE;
  const uint32_t sBar = sEpi + Cfg::EPI_BYTES;
  uint8_t* bar_ptr = base_ptr + (sBar - base);
  // 8-byte barriers and words: full[8], empty[8], tfull[2], tempty[2], done, skdone,
  // the TMEM base address, the abort flag, the two producers' issued-stage counts
  // (pair error drain); then the CLC ring (sfull, sempty, 16-byte responses)
  const uint32_t bar_full = sBar;
  const uint32_t bar_empty = sBar + 64;
  const uint32_t bar_tfull = sBar + 128;
  const uint32_t bar_tempty = sBar + 144;
  const uint32_t bar_done = sBar + 160;
  const uint32_t bar_skdone = sBar + 168;               // stream-K: partial written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_ptr + 176);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(bar_ptr + 180);
  const uint32_t abort_addr = sBar + 180;
  // issued[r] = k-block stages the producer of in-pair rank r issued (rank 1 writes
  // its count into the leader's word over DSMEM)
  volatile uint32_t* issued_words = reinterpret_cast<volatile uint32_t*>(bar_ptr + 184);
  const uint32_t issued_addr = sBar + 184;
  const uint32_t bar_sfull = sBar + 192;                // CLC_SLOTS (≤ 8)
  const uint32_t bar_sempty = sBar + 256;               // CLC_SLOTS
  const uint32_t clc_resp = sBar + 320;                 // CLC_SLOTS × 16 B

  const uint32_t warp = warp_id(), lane = lane_id();
  // In-pair rank (0 = the pair's MMA leader).
  const uint32_t rank = (CG == 2) ? cluster_ctarank() : 0u;
  const uint32_t peer = rank ^ 1u;

  if (warp == 0 && lane == 0) {
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (uint32_t a = 0; a < 2; ++a) {
      mbar_init(bar_tfull + 8 * a, 1);
      // every epilogue warp of the pair hands the accumulator back to the leader
      mbar_init(bar_tempty + 8 * a, Cfg::EPI_WARPS * CG);
    }
    for (uint32_t a = 0; a < Cfg::CLC_SLOTS; ++a) {
      // leader: the try_cancel response (tx); peer: the leader's forwarding arrive
      mbar_init(bar_sfull + 8 * a, 1);
      // slot release: every consumer of the pair arrives on the leader's barrier
      mbar_init(bar_sempty + 8 * a, Cfg::SCHED_CONSUMERS * CG);
    }
    mbar_init(bar_done, 1);
    mbar_init(bar_skdone, Cfg::EPI_WARPS);
    *abort_flag = 0u;
    issued_words[0] = 0u;
    issued_words[1] = 0u;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc<CG>(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish<CG>();
  }
  tc_fence_before();
  if constexpr (CG == 2) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The set-up above touches no global memory, so with programmatic dependent launch
  // it overlaps the previous kernel's tail; every global access comes after this wait.
  griddep_wait();
  griddep_launch_dependents();

  // A role that gives up raises the abort flag of its own CTA and, in a pair, of the
  // peer too, so the other CTA's waits stop early and both CTAs agree at teardown
  // that the pair aborted. (The peer is alive: fail() is only called before the
  // teardown cluster barrier, or by the leader's drain while the peer waits in the
  // second one.)
  auto fail = [&](uint32_t code) {
    *abort_flag = 1u;
    if constexpr (CG == 2) st_shared_cluster_u32(mapa_shared(abort_addr, peer), 1u);
    if (p.status) atomicOr(p.status, code | ST_ABORTED);
  };

  // ---- TMEM slots: tile `it`, MMA h -> slot; each use of a slot flips its phase ----
  // NH = 1: tiles alternate between the two slots (double buffering).
  // NH = 2: every tile uses both slots, MMA h in slot h.
  auto acc_slot = [](uint32_t it, int h) -> uint32_t { return NH == 1 ? (it & 1u) : uint32_t(h); };
  auto acc_use = [](uint32_t it) -> uint32_t { return NH == 1 ? (it >> 1) : it; };

  // ---- tile id -> (block-row, block-col) ----
  auto tile_coords = [&](uint32_t tile, uint32_t& bm, uint32_t& bn) {
    tile_to_bmn(tile, p.m_tiles, p.n_tiles, p.group_m, bm, bn);
  };

  // ---- tile sequence shared by every role ----
  // SCHED_STATIC: cluster c takes tiles c, c + G, c + 2G, ... (G = clusters in grid)
  // SCHED_CLC   : tile = this cluster's own index first, then whatever the
  //               leader's try_cancel returns (forwarded to the peer)
  const uint32_t first_tile = blockIdx.x / CG;
  const uint32_t tile_stride = gridDim.x / CG;
  const uint32_t leader_sempty0 = (CG == 2) ? mapa_shared(bar_sempty, 0) : bar_sempty;

  // Consumer side of the CLC ring: wait for slot, decode, release it to the leader.
  // Returns false when the grid is exhausted (tile unchanged) or on abort.
  // The release must follow the read of the response: the scheduler rewrites the
  // slot (try_cancel in the leader, a DSMEM store in the peer) as soon as all 10 * CG
  // consumers have released it. A relaxed arrive alone does not order the earlier
  // ld.shared, so a consumer whose load waited behind long-latency stores (an
  // epilogue warp with multimem stores to other GPUs in flight) could decode the
  // slot's NEXT response, drop out of the tile sequence and leave the pair's TMEM
  // hand-off waiting; fence_release_smem() orders the load without waiting for the
  // warp's global stores.
  uint32_t sched_slot = 0, sched_phase = 0;
  auto clc_next = [&](uint32_t& tile) -> bool {
    if (!mbar_wait<CG == 2>(bar_sfull + 8 * sched_slot, sched_phase, p.wait_ns, abort_flag)) {
      fail(ST_SCHED);
      return false;
    }
    uint32_t x = 0;
    const bool got = clc_decode(clc_resp + 16 * sched_slot, x);
    if constexpr (CG == 1) {
      mbar_arrive(bar_sempty + 8 * sched_slot);  // release.cta: orders the read
    } else {
      fence_release_smem();
      mbar_arrive_cluster_relaxed(leader_sempty0 + 8 * sched_slot);
    }
    if (++sched_slot == Cfg::CLC_SLOTS) { sched_slot = 0; sched_phase ^= 1u; }
    if (got) tile = x / CG;
    return got;
  };

  // Next tile after `tile`, fetched by every role at the START of its current tile
  // so that with CLC the ring slot is released a whole tile before the scheduler
  // needs it again (at small K a tile is only a few pipeline stages long).
  auto fetch_next = [&](uint32_t tile, uint32_t& next) -> bool {
    if constexpr (SCHED == SCHED_CLC) {
      next = tile;
      return clc_next(next);
    } else {
      next = tile + tile_stride;
      return next < p.num_tiles;
    }
  };

  // ---- stream-K: worker w owns iterations [w*T/W, (w+1)*T/W) of the T = tiles x
  // k-blocks iterations, in tile order. A worker's range ends inside at most one
  // tile (its PARTIAL item, done first so no worker waits before writing) and
  // starts inside at most one (its LAST item). ----
  const uint32_t n_workers = gridDim.x / CG;
  const uint32_t worker = blockIdx.x / CG;
  const uint64_t total_iters = uint64_t(p.num_tiles) * p.k_blocks;
  auto sk_start = [&](uint32_t w) -> uint64_t { return total_iters * w / n_workers; };
  const uint64_t my_begin = sk_start(worker), my_end = sk_start(worker + 1);
  const bool sk_any = my_begin < my_end;
  const uint32_t t_first = sk_any ? uint32_t(my_begin / p.k_blocks) : 0u;
  const uint32_t t_last = sk_any ? uint32_t((my_end - 1) / p.k_blocks) : 0u;
  const bool last_partial = sk_any && (my_end % p.k_blocks) != 0;
  const uint32_t n_items = sk_any ? t_last - t_first + 1 : 0u;
  auto sk_item = [&](uint32_t i, WorkItem& it) -> bool {
    if (i >= n_items) return false;
    const uint32_t t = last_partial ? (i == 0 ? t_last : t_first + i - 1) : t_first + i;
    const uint64_t tb = uint64_t(t) * p.k_blocks, te = tb + p.k_blocks;
    it.tile = t;
    it.kb0 = uint32_t((my_begin > tb ? my_begin : tb) - tb);
    it.kb1 = uint32_t((my_end < te ? my_end : te) - tb);
    it.kind = it.kb1 < p.k_blocks ? ITEM_PARTIAL : (it.kb0 > 0 ? ITEM_LAST : ITEM_FULL);
    it.idx = i;
    return true;
  };
  // The worker whose range holds iteration i.
  auto sk_owner = [&](uint64_t i) -> uint32_t {
    uint32_t w = uint32_t(i * n_workers / total_iters);
    while (w + 1 < n_workers && sk_start(w + 1) <= i) ++w;
    while (w > 0 && sk_start(w) > i) --w;
    return w;
  };

  auto first_item = [&](WorkItem& it) -> bool {
    if constexpr (SCHED == SCHED_STREAMK) {
      return sk_item(0, it);
    } else {
      it = WorkItem{first_tile, 0u, p.k_blocks, ITEM_FULL, 0u};
      return first_tile < p.num_tiles;
    }
  };
  auto next_item = [&](const WorkItem& cur, WorkItem& nxt) -> bool {
    if constexpr (SCHED == SCHED_STREAMK) {
      return sk_item(cur.idx + 1, nxt);
    } else {
      uint32_t nt;
      const bool more = fetch_next(cur.tile, nt);
      nxt = WorkItem{nt, 0u, p.k_blocks, ITEM_FULL, cur.idx + 1};
      return more;
    }
  };

  if (warp == 0) {
    // =============================== TMA producer ===============================
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      const uint64_t hint_a = (p.l2_policy & 1u)   ? policy_evict_last()
                              : (p.l2_policy & 8u) ? policy_evict_first()
                                                   : policy_evict_normal();
      const uint64_t hint_b = (p.l2_policy & 2u)    ? policy_evict_first()
                              : (p.l2_policy & 16u) ? policy_evict_last()
                                                    : policy_evict_normal();
      const uint32_t leader_full0 = (CG == 2) ? mapa_shared(bar_full, 0) : bar_full;
      if (!p.fault_inject) {
        WorkItem cur;
        bool more = first_item(cur);
        while (more && ok) {
          WorkItem nxt;
          const bool next_more = next_item(cur, nxt);
          uint32_t bm, bn;
          tile_coords(cur.tile, bm, bn);
          const int32_t a_row = int32_t((bm * CG + rank) * Cfg::BM);
          // rows of this CTA's share of MMA h: bn*BN + h*MMA_N + rank*B_HALF_ROWS
          const int32_t b_row = int32_t(bn * Cfg::BN + rank * Cfg::B_HALF_ROWS);
          // this CTA's boxes of k-block kb, into L2 only; boxes that reach past an edge
          // of A or B are left to the loads
          auto prefetch = [&](uint32_t kb) {
#pragma unroll
            for (int at = 0; at < Cfg::ATOMS; ++at) {
              const uint32_t x = kb * Cfg::BK + at * Cfg::ATOM_K;
              if (x + Cfg::ATOM_K > p.K) break;
              if (uint32_t(a_row) + Cfg::BM <= p.M) tma_prefetch_2d(&tmA, int32_t(x), a_row);
#pragma unroll
              for (int h = 0; h < NH; ++h) {
                const uint32_t r = uint32_t(b_row + h * Cfg::MMA_N);
                if (r + Cfg::B_HALF_ROWS <= p.N) tma_prefetch_2d(&tmB, int32_t(x), int32_t(r));
              }
            }
          };
          if (p.prefetch_k) {
            const uint32_t pend = min(cur.kb1, cur.kb0 + p.prefetch_k);
            for (uint32_t kb = cur.kb0 + S; kb < pend; ++kb) prefetch(kb);
          }
          for (uint32_t kb = cur.kb0; kb < cur.kb1; ++kb) {
            if (!mbar_wait(bar_empty + 8 * stage, phase ^ 1u, p.wait_ns, abort_flag)) {
              fail(ST_PRODUCER_EMPTY);
              ok = false;
              break;
            }
            const int32_t kx = int32_t(kb * Cfg::BK);
            if constexpr (CG == 1) {
              mbar_arrive_expect_tx(bar_full + 8 * stage, Cfg::STAGE);
#pragma unroll
              for (int at = 0; at < Cfg::ATOMS; ++at) {
                const int32_t x = kx + at * Cfg::ATOM_K;
                tma_load_2d(sA + stage * Cfg::A_STAGE + at * Cfg::A_ATOM, &tmA, x, a_row, bar_full + 8 * stage, hint_a);
#pragma unroll
                for (int h = 0; h < NH; ++h)
                  tma_load_2d(sB + stage * Cfg::B_STAGE + at * Cfg::B_ATOM + h * Cfg::B_HALF, &tmB, x,
                              b_row + h * Cfg::MMA_N, bar_full + 8 * stage, hint_b);
              }
            } else {
              // Both CTAs' bytes are credited to the leader's full barrier; only the
              // leader arms it (a peer credit that lands first leaves the tx count
              // negative but cannot complete the phase without the leader's arrive).
              if (rank == 0) mbar_arrive_expect_tx(bar_full + 8 * stage, 2 * Cfg::STAGE);
              const uint32_t lf = leader_full0 + 8 * stage;
#pragma unroll
              for (int at = 0; at < Cfg::ATOMS; ++at) {
                const int32_t x = kx + at * Cfg::ATOM_K;
                tma_load_2d_pair(sA + stage * Cfg::A_STAGE + at * Cfg::A_ATOM, &tmA, x, a_row, lf, hint_a);
#pragma unroll
                for (int h = 0; h < NH; ++h)
                  tma_load_2d_pair(sB + stage * Cfg::B_STAGE + at * Cfg::B_ATOM + h * Cfg::B_HALF, &tmB, x,
                                   b_row + h * Cfg::MMA_N, lf, hint_b);
              }
            }
            if (p.prefetch_k && kb + p.prefetch_k < cur.kb1) prefetch(kb + p.prefetch_k);
            ++issued;
            if (++stage == S) { stage = 0; phase ^= 1u; }
          }
          if (!ok) break;
          cur = nxt;
          more = next_more;
        }
      }
      if constexpr (CG == 1) {
        if (!ok || *abort_flag) {
          // Error path: wait (bounded) for the loads this CTA still has in flight so
          // that no TMA write lands after the CTA's shared memory is released. Every
          // stage before the last S was consumed by the MMA, so only the last S can
          // still be in flight.
          const uint32_t first = issued > S ? issued - S : 0u;
          for (uint32_t i = first; i < issued; ++i) {
            if (!mbar_wait_bounded(bar_full + 8 * (i % S), (i / S) & 1u, p.wait_ns)) {
              fail(ST_DRAIN);
              break;
            }
          }
        }
      } else {
        // The pair's loads are credited to the leader's full barriers, so the leader
        // drains both CTAs' copies after the roles have stopped (teardown below). It
        // needs both counts; the store is ordered before the teardown cluster barrier.
        if (rank == 0) issued_words[0] = issued;
        else st_shared_cluster_u32(mapa_shared(issued_addr + 4, 0), issued);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ============================ MMA issuer (leader) ============================
    if (lane == 0 && rank == 0) {
      uint32_t stage = 0, phase = 0, tile_iter = 0;
      bool ok = true;
      WorkItem cur;
      bool more = first_item(cur);
      while (more && ok) {
        WorkItem nxt;
        const bool next_more = next_item(cur, nxt);
        for (uint32_t kb = cur.kb0; kb < cur.kb1; ++kb) {
          // TMA completion on the mbarrier makes the stage visible to the MMA; no
          // tcgen05 fence is needed between this wait and the MMAs.
          if (!mbar_wait(bar_full + 8 * stage, phase, p.wait_ns, abort_flag)) {
            fail(ST_MMA_FULL);
            ok = false;
            break;
          }
          const uint32_t a0 = sA + stage * Cfg::A_STAGE;
          const uint32_t b0 = sB + stage * Cfg::B_STAGE;
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            const uint32_t slot = acc_slot(tile_iter, h);
            if (kb == cur.kb0) {
              // the slot's previous contents must have been drained by the epilogue
              if (!mbar_wait(bar_tempty + 8 * slot, (acc_use(tile_iter) & 1u) ^ 1u, p.wait_ns,
                             abort_flag)) {
                fail(ST_MMA_TMEM_EMPTY);
                ok = false;
                break;
              }
              tc_fence_after();
            }
            const uint32_t d_tmem = tmem_base + slot * Cfg::MMA_N;
#pragma unroll
            for (uint32_t k = 0; k < Cfg::KSTEPS; ++k) {
              const uint32_t a_k = a0 + (k / 4) * Cfg::A_ATOM + 32u * (k % 4);
              const uint32_t b_k = b0 + (k / 4) * Cfg::B_ATOM + h * Cfg::B_HALF + 32u * (k % 4);
              umma<CG, Cfg::KIND>(d_tmem, sdesc_k_sw128(a_k), sdesc_k_sw128(b_k), Cfg::IDESC,
                                  ((kb - cur.kb0) | k) != 0u ? 1u : 0u);
            }
            if (kb + 1 == cur.kb1) {
              // Slot h is final once these MMAs complete: signal it now, so with two
              // MMAs per tile the epilogue drains slot 0 while the last MMAs into
              // slot 1 run.
              if constexpr (CG == 1) umma_commit<1>(bar_tfull + 8 * slot);
              else umma_commit_pair(bar_tfull + 8 * slot, uint16_t(3u));
            }
          }
          if (!ok) break;
          // frees this stage in both CTAs once the MMAs above have read it
          if constexpr (CG == 1) umma_commit<1>(bar_empty + 8 * stage);
          else umma_commit_pair(bar_empty + 8 * stage, uint16_t(3u));
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        ++tile_iter;
        cur = nxt;
        more = next_more;
      }
      // Every MMA this thread issued must retire before TMEM is released.
      umma_commit<CG>(bar_done);
      if (!mbar_wait_bounded(bar_done, 0, p.wait_ns)) fail(ST_DRAIN);
    } else if (SCHED == SCHED_CLC && lane == 0 && rank != 0) {
      // the peer's MMA warp has no MMA work but still consumes the schedule
      uint32_t tile = first_tile;
      bool more = tile < p.num_tiles;
      while (more) more = clc_next(tile);
    }
    __syncwarp();
  } else if (warp == 2) {
    // ============================== CLC scheduler ==============================
    if constexpr (SCHED == SCHED_CLC) {
      if (lane == 0 && rank == 0 && first_tile < p.num_tiles) {
        uint32_t slot = 0, ph = 0;
        const uint32_t peer_sfull0 = (CG == 2) ? mapa_shared(bar_sfull, 1) : 0u;
        const uint32_t peer_resp0 = (CG == 2) ? mapa_shared(clc_resp, 1) : 0u;
        while (true) {
          // every consumer of both CTAs has read the slot's previous response
          // (acquire.cluster pairs with the peers' fence_release_smem + arrive)
          if (!mbar_wait<CG == 2>(bar_sempty + 8 * slot, ph ^ 1u, p.wait_ns, abort_flag)) {
            fail(ST_SCHED);
            break;
          }
          mbar_arrive_expect_tx(bar_sfull + 8 * slot, 16);
          clc_try_cancel(clc_resp + 16 * slot, bar_sfull + 8 * slot);
          // The response is an async write into this CTA's shared memory: wait for it
          // even when the CTA is aborting, so that it cannot land after the CTA exits.
          if (!mbar_wait_bounded(bar_sfull + 8 * slot, ph, p.wait_ns)) {
            fail(ST_SCHED);
            break;
          }
          uint32_t x;
          const bool got = clc_decode(clc_resp + 16 * slot, x);
          if constexpr (CG == 2) {
            // forward the 16-byte response to the peer, then release it there
            uint32_t r0, r1, r2, r3;
            ld_shared_v4(clc_resp + 16 * slot, r0, r1, r2, r3);
            st_shared_cluster_v4(peer_resp0 + 16 * slot, r0, r1, r2, r3);
            mbar_arrive_cluster(peer_sfull0 + 8 * slot);
          }
          if (!got) break;  // grid exhausted: a failed request ends the schedule
          if (++slot == Cfg::CLC_SLOTS) { slot = 0; ph ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ================================ epilogue ================================
    const uint32_t q = (warp - 4) & 3u;  // TMEM lane quarter == warp id % 4
    const uint32_t e = (warp - 4) >> 2;  // column half of each slot
    float scale = 1.0f;
    if (p.scale_a) scale *= __ldg(p.scale_a);
    if (p.scale_b) scale *= __ldg(p.scale_b);
    const uint32_t my_buf = sEpi + (warp - 4) * Cfg::EPI_BUF;
    const bool c_hint = (p.l2_policy & 4u) != 0u;
    const uint64_t hint_c = policy_evict_first();
    const uint32_t leader_tempty0 = (CG == 2) ? mapa_shared(bar_tempty, 0) : bar_tempty;
    uint32_t tile_iter = 0;
    WorkItem cur;
    bool more = first_item(cur);
    bool ok = true;
    while (more && ok) {
      WorkItem nxt;
      bool next_more;
      if constexpr (SCHED == SCHED_CLC) {
        uint32_t next = cur.tile;
        bool got = false;
        if (lane == 0) got = clc_next(next);
        next_more = __shfl_sync(0xffffffffu, got ? 1u : 0u, 0) != 0u;
        nxt = WorkItem{__shfl_sync(0xffffffffu, next, 0), 0u, p.k_blocks, ITEM_FULL, cur.idx + 1};
      } else {
        next_more = next_item(cur, nxt);
      }
      uint32_t bm, bn;
      tile_coords(cur.tile, bm, bn);
      const int32_t row0 = int32_t((bm * CG + rank) * Cfg::BM + 32 * q);
#pragma unroll 1
      for (int h = 0; h < NH; ++h) {
        const uint32_t slot = acc_slot(tile_iter, h);
        const uint32_t par = acc_use(tile_iter) & 1u;
        uint32_t okw = 0;
        if (lane == 0) {
          if constexpr (NH == 1) {
            // Double-buffered accumulator: the drain is off the MMA's critical path,
            // so sleep between polls (bounded by the same deadline and abort flag).
            const uint64_t t0 = globaltimer_ns();
            bool done;
            while (!(done = mbar_try_wait(bar_tfull + 8 * slot, par))) {
              if (*abort_flag || globaltimer_ns() - t0 > p.wait_ns) break;
              __nanosleep(1000);
            }
            okw = done ? 1u : 0u;
          } else {
            // Single-buffered accumulator: the next tile's MMAs wait for this drain,
            // so wake on the barrier itself rather than on a sleep timer.
            okw = mbar_wait(bar_tfull + 8 * slot, par, p.wait_ns, abort_flag) ? 1u : 0u;
          }
        }
        okw = __shfl_sync(0xffffffffu, okw, 0);
        if (!okw) {
          if (lane == 0) fail(ST_EPI_TMEM_FULL);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t_row = tmem_base + ((32u * q) << 16) + slot * Cfg::MMA_N;
        const uint32_t c0 = e * Cfg::EPI_CHUNKS_PER_WARP;
        // Read every TMEM column this warp owns in the slot, then release the slot
        // before converting: the next tile's MMAs into it can start meanwhile.
        uint32_t r[Cfg::EPI_CHUNKS_PER_WARP][Cfg::EPI_COLS];
#pragma unroll
        for (int cc = 0; cc < Cfg::EPI_CHUNKS_PER_WARP; ++cc) {
#pragma unroll
          for (int x = 0; x < Cfg::EPI_COLS / 32; ++x) {
            uint32_t (&rr)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[cc][32 * x]);
            tmem_ld_x32(t_row + (c0 + cc) * Cfg::EPI_COLS + 32 * x, rr);
          }
        }
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (CG == 1) mbar_arrive(bar_tempty + 8 * slot);
          else mbar_arrive_cluster_relaxed(leader_tempty0 + 8 * slot);  // TMEM read: relaxed
        }
        if constexpr (SCHED == SCHED_STREAMK) {
          // Each thread owns EPI_VALS consecutive fp32 values (its row, its columns of
          // the slot); the workspace stores them thread-major so that every access of
          // a warp is 512 contiguous bytes: float4 j of warp w4, lane l at
          // (w4*J + j)*32 + l, J = EPI_VALS / 4.
          constexpr uint32_t J = Cfg::EPI_VALS / 4;
          const uint32_t w4 = warp - 4;
          if (cur.kind == ITEM_PARTIAL) {
            float4* ws = reinterpret_cast<float4*>(p.sk_work) + size_t(worker * CG + rank) * (Cfg::SK_FLOATS / 4);
#pragma unroll
            for (uint32_t j = 0; j < J; ++j) {
              const uint32_t f = 4 * j, cc = f / Cfg::EPI_COLS, x = f % Cfg::EPI_COLS;
              __stcg(ws + (w4 * J + j) * 32 + lane,
                     make_float4(__uint_as_float(r[cc][x]), __uint_as_float(r[cc][x + 1]),
                                 __uint_as_float(r[cc][x + 2]), __uint_as_float(r[cc][x + 3])));
            }
            __threadfence();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_skdone);
            if (warp == 4 && lane == 0) {
              // every epilogue warp wrote its part: publish the partial for this launch
              if (mbar_wait(bar_skdone, 0, p.wait_ns, abort_flag))
                st_release_gpu(p.sk_flags + worker * CG + rank, p.sk_epoch);
              else
                fail(ST_STREAMK);
            }
            continue;  // a partial tile stores no C
          }
          if (cur.kind == ITEM_LAST) {
            // add the partial sums of every worker that owns an earlier part of the tile
            const uint32_t w_lo = sk_owner(uint64_t(cur.tile) * p.k_blocks);
            for (uint32_t w2 = w_lo; w2 < worker && ok; ++w2) {
              if (sk_start(w2) == sk_start(w2 + 1)) continue;  // empty range
              const uint32_t* flag = p.sk_flags + w2 * CG + rank;
              uint32_t okf = 1;
              if (lane == 0) {
                const uint64_t t0 = globaltimer_ns();
                while (ld_acquire_gpu(flag) != p.sk_epoch) {
                  if (*abort_flag || globaltimer_ns() - t0 > p.wait_ns) { okf = 0; break; }
                  __nanosleep(256);
                }
              }
              okf = __shfl_sync(0xffffffffu, okf, 0);
              if (!okf) {
                if (lane == 0) fail(ST_STREAMK);
                ok = false;
                break;
              }
              const float4* src =
                  reinterpret_cast<const float4*>(p.sk_work) + size_t(w2 * CG + rank) * (Cfg::SK_FLOATS / 4);
#pragma unroll
              for (uint32_t j = 0; j < J; ++j) {
                const uint32_t f = 4 * j, cc = f / Cfg::EPI_COLS, x = f % Cfg::EPI_COLS;
                const float4 v = __ldcg(src + (w4 * J + j) * 32 + lane);
                r[cc][x] = __float_as_uint(__uint_as_float(r[cc][x]) + v.x);
                r[cc][x + 1] = __float_as_uint(__uint_as_float(r[cc][x + 1]) + v.y);
                r[cc][x + 2] = __float_as_uint(__uint_as_float(r[cc][x + 2]) + v.z);
                r[cc][x + 3] = __float_as_uint(__uint_as_float(r[cc][x + 3]) + v.w);
              }
            }
            if (!ok) break;
          }
        }
#pragma unroll
        for (int cc = 0; cc < Cfg::EPI_CHUNKS_PER_WARP; ++cc) {
          uint32_t w[32];
          if constexpr (Cfg::CD_BYTES == 4) {
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(__uint_as_float(r[cc][i]) * scale);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float x0 = __uint_as_float(r[cc][2 * i]) * scale;
              const float x1 = __uint_as_float(r[cc][2 * i + 1]) * scale;
              if constexpr (CD == DT_BF16) w[i] = pack_bf16x2(x0, x1);
              else w[i] = pack_f16x2(x0, x1);
            }
          }
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
          const uint32_t sb = my_buf;
          const uint32_t row_addr = sb + lane * 128u;
#pragma unroll
          for (uint32_t j = 0; j < 8; ++j) {
            st_shared_v4(row_addr + ((j ^ (lane & 7u)) << 4), w[4 * j], w[4 * j + 1], w[4 * j + 2],
                         w[4 * j + 3]);
          }
          fence_proxy_async_shared();
          __syncwarp();
          const uint32_t col0 = bn * Cfg::BN + h * Cfg::MMA_N + (c0 + cc) * Cfg::EPI_COLS;
          if (lane == 0) {
            if (uint32_t(row0) < p.M && col0 < p.N) {
              if (c_hint) tma_store_2d_hint(&tmC, sb, int32_t(col0), row0, hint_c);
              else tma_store_2d(&tmC, sb, int32_t(col0), row0);
            }
            bulk_commit();
          }
          if (p.gather_mode != GATHER_OFF) {
            // The staged 32 x 128-byte chunk again, read row-contiguously (8 lanes per
            // row, 16 bytes each) and stored into every GPU's gathered C; the host
            // checked that N, the pitch and the column offset keep 16-byte chunks
            // whole and aligned.
            const uint32_t j = lane & 7u;
            const uint32_t col = col0 + j * (16u / Cfg::CD_BYTES);
#pragma unroll
            for (uint32_t i = 0; i < 8; ++i) {
              const uint32_t rr = 4u * i + (lane >> 3);
              uint32_t x0, x1, x2, x3;
              ld_shared_v4(sb + rr * 128u + ((j ^ (rr & 7u)) << 4), x0, x1, x2, x3);
              const uint32_t grow = uint32_t(row0) + rr;
              if (grow < p.M && col < p.N) {
                const uint64_t off = (uint64_t(grow) * p.gather_ld + p.gather_col + col) * Cfg::CD_BYTES;
                if (p.gather_mode == GATHER_MULTICAST) {
                  multimem_st_v4(reinterpret_cast<uint64_t>(p.gather) + off, x0, x1, x2, x3);
                } else {
                  const uint64_t* bases = reinterpret_cast<const uint64_t*>(p.gather);
                  for (uint32_t g = 0; g < p.gather_peers; ++g)
                    *reinterpret_cast<uint4*>(bases[g] + off) = make_uint4(x0, x1, x2, x3);
                }
              }
            }
          }
        }
      }
      if (!ok) break;
      ++tile_iter;
      cur = nxt;
      more = next_more;
    }
    if (lane == 0) bulk_wait<0>();
    // gathered stores to other GPUs are performed before the kernel is seen complete
    if (p.gather_mode != GATHER_OFF) __threadfence_system();
    __syncwarp();
  }

  // ---- teardown: every role has left its loop; release TMEM ----
  tc_fence_before();
  if constexpr (CG == 2) {
    cluster_sync();
    // Error drain of the pair. Both CTAs' TMA loads are credited to the leader's full
    // barriers, so a CTA cannot see its own loads land. After an abort in either CTA,
    // the leader's producer thread waits for every stage still in flight, completing
    // the phases whose bytes will never come, before either CTA leaves: at most the
    // last S stages of either producer can be unconsumed (a producer issues stage i
    // only after the MMA consumed stage i - S, which needed both producers' bytes).
    // fail() raises both CTAs' flags before the barrier above, so both CTAs agree on
    // the extra barrier below.
    if (*abort_flag) {
      if (warp == 0 && lane == 0 && rank == 0) {
        const uint32_t il = issued_words[0], ip = issued_words[1];
        const uint32_t hi = il > ip ? il : ip;
        for (uint32_t i = hi > S ? hi - S : 0u; i < hi; ++i) {
          const uint32_t bar = bar_full + 8 * (i % S);
          // A phase with a missing half cannot have completed, so the fix-ups below
          // only touch phases still open: the leader never armed stage i (wait for
          // the peer's bytes alone), or the peer never loaded it (take its bytes off).
          if (i >= il) mbar_arrive_expect_tx(bar, Cfg::STAGE);
          else if (i >= ip) mbar_complete_tx(bar, Cfg::STAGE);
          if (!mbar_wait_bounded(bar, (i / S) & 1u, p.wait_ns)) {
            fail(ST_DRAIN);
            break;
          }
        }
      }
      cluster_sync();
    }
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<CG>(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace b200
