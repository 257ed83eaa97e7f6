// sm100_ptx.cuh — inline-PTX primitives for Blackwell (sm_100a).
//
// This is the B200 replacement for the reference's three device headers:
//   include/common/mbarrier.cuh:17-84  (mbarrier init/arrive/expect_tx/wait, TMA 2D load/store)
//   include/common/gmma.cuh:30-199     (wgmma smem descriptors and wgmma.mma_async)
//   include/common/cluster.cuh:20-98   (cluster rank, mapa, cluster barrier, remote arrive)
// On sm_100a the tensor-core path is tcgen05: the MMA is issued by a single thread,
// the accumulator lives in Tensor Memory (TMEM), completion is signalled to an
// mbarrier with tcgen05.commit, and the epilogue reads TMEM with tcgen05.ld.
//
// Differences from the reference that matter for safety on a shared GPU:
//   * every mbarrier wait is bounded by %globaltimer and by a CTA-wide abort flag,
//     so a protocol error becomes an error code instead of a hung GPU
//     (the reference spins forever: mbarrier.cuh:37-47);
//   * every TMA load here is a plain unicast copy into the issuing CTA's own shared
//     memory, so the same binary can run on every GPU of a box; the one cluster-wide
//     signal is the pair kernel's tcgen05.commit (umma_commit_pair), which moves no
//     data.
#pragma once

#include <cuda.h>
#include <cstdint>

namespace b200 {

// ---------------------------------------------------------------------------------
// generic helpers
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31; }

// ---------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes mbarrier.init visible to the async proxy (TMA, tcgen05) and to the cluster.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// Arrive on an mbarrier that lives in another CTA of the cluster (address from mapa).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}

// Programmatic dependent launch: wait until every prerequisite grid of the stream has
// completed and its memory is visible (before this kernel's first global access), and
// allow the next kernel of the stream to be scheduled once all CTAs of this grid ran
// launch_dependents (its CTAs then do their set-up on SMs this grid leaves free and
// wait in their own griddepcontrol.wait).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Relaxed remote arrive. On its own it orders nothing: the memory model lets it
// become visible before this thread's earlier loads have read their data. Two uses:
//   * a drained TMEM accumulator: tcgen05.wait::ld has returned, so the TMEM reads
//     are complete, and the arrive only has to follow them (no release needed);
//   * after fence_release_smem(): the fence orders this thread's earlier shared::cta
//     accesses (the ld.shared of a CLC response) before the arrive.
// A release.cluster arrive would also wait for this thread's earlier global and bulk
// stores (an epilogue warp's TMA stores, or its multimem stores to other GPUs) to
// become visible cluster-wide: measured ~1 us per arrive, which stalled the pair
// kernels' MMA and scheduler.
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}

// Release fence restricted to shared::cta: this thread's earlier shared::cta loads
// and stores are ordered before its following (relaxed) mbarrier arrive on a
// shared::cluster barrier, without waiting for its global or bulk stores. Paired
// with an acquire.cluster wait on that barrier, it makes "I have read this slot"
// safe to act on: the slot's next writer cannot overtake the read.
__device__ __forceinline__ void fence_release_smem() {
  asm volatile("fence.release.sync_restrict::shared::cta.cluster;" ::: "memory");
}

// Take `bytes` off the pending transaction count of the current phase, as if that
// many bytes of an async copy had landed. Used only on the error path, to complete
// a phase whose expected bytes will never come.
__device__ __forceinline__ void mbar_complete_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.complete_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait with a suspend-time hint: a waiting thread is parked by the hardware
// until the phase completes or about `ns` nanoseconds pass, instead of spinning
// and taking issue slots from the producer and MMA warps.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return done != 0;
}

// Same, with acquire semantics at cluster scope: for barriers that another CTA of
// the cluster completes with a release.cluster arrive after writing our smem.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return done != 0;
}

constexpr uint32_t kSuspendHintNs = 100000u;  // re-check abort / deadline every ~100 us

// Bounded wait. Returns true when the phase with `parity` completed; false when
// either `limit_ns` of %globaltimer elapsed or another role of the CTA raised
// `*abort`. The caller turns `false` into an error code and leaves its loop.
template <bool kClusterScope = false>
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t limit_ns,
                                          volatile uint32_t* abort) {
  if (kClusterScope ? mbar_try_wait_cluster(bar, parity, 0u) : mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (kClusterScope ? mbar_try_wait_cluster(bar, parity, kSuspendHintNs)
                      : mbar_try_wait_hint(bar, parity, kSuspendHintNs))
      return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// Bounded wait that ignores the abort flag: used on the teardown path, where a
// role drains its own in-flight work after the CTA already aborted.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_hint(bar, parity, kSuspendHintNs)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// GPU-scope acquire load / release store of a flag in global memory (stream-K
// partial-tile hand-off between CTAs).
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* ptr) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* ptr, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

// ---------------------------------------------------------------------------------
// cluster
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// Translate a local shared::cta address into the shared::cluster address of the
// same offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void st_shared_cluster_v4(uint32_t cluster_addr, uint32_t a, uint32_t b,
                                                     uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "r"(a), "r"(b),
               "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ void st_shared_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_shared_cluster_u32(uint32_t cluster_addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
  return v;
}

__device__ __forceinline__ void ld_shared_v4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c,
                                             uint32_t& d) {
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr)
               : "memory");
}

// ---------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor): unicast loads and stores only
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* m, int32_t x,
                                            int32_t y, uint32_t bar, uint64_t hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(m), "r"(x), "r"(y), "r"(bar), "l"(hint)
      : "memory");
}

// L2 prefetch of one box of a tiled tensor map: the TMA unit brings the box into L2
// (no shared memory, no barrier), so a later load of it is an L2 hit.
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* m, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(m), "r"(x), "r"(y)
               : "memory");
}

// Pair form for cta_group::2: the data lands in this CTA's shared memory, the
// completion bytes are credited to `bar`, which may be the leader CTA's barrier.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* m, int32_t x,
                                                 int32_t y, uint32_t cluster_bar, uint64_t hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(m), "r"(x), "r"(y), "r"(cluster_bar), "l"(hint)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, uint32_t src, int32_t x,
                                             int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(m),
               "r"(x), "r"(y), "r"(src)
               : "memory");
}

// Same, with an L2 cache policy for the written lines.
__device__ __forceinline__ void tma_store_2d_hint(const CUtensorMap* m, uint32_t src, int32_t x, int32_t y,
                                                  uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group.L2::cache_hint [%0, {%1, %2}], [%3], %4;" ::"l"(m),
      "r"(x), "r"(y), "r"(src), "l"(policy)
      : "memory");
}

// One 16-byte store to a multicast (NVLS) address: the NVSwitch delivers it to the
// same offset of every GPU bound to the multicast object. Bitwise: the four words are
// moved as they are (typed f32 only because the instruction names a type).
__device__ __forceinline__ void multimem_st_v4(uint64_t addr, uint32_t a, uint32_t b, uint32_t c,
                                               uint32_t d) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr),
               "f"(__uint_as_float(a)), "f"(__uint_as_float(b)), "f"(__uint_as_float(c)),
               "f"(__uint_as_float(d))
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Generic-proxy shared-memory writes -> visible to the async proxy (TMA store).
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// L2 cache-policy descriptors for the .L2::cache_hint operand.
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------------
// tcgen05: Tensor Memory
// ---------------------------------------------------------------------------------
template <int CG>
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
  else
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_relinquish() {
  if constexpr (CG == 1)
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  else
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
  else
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------------
// tcgen05: descriptors
// ---------------------------------------------------------------------------------
// Shared-memory matrix descriptor (tcgen05 format) for a K-major operand tile laid
// out by a TMA load with SWIZZLE_128B: rows of 128 bytes, 8-row swizzle atoms of
// 1024 bytes stacked along M/N.
//   bits  0-13  start address >> 4
//   bits 16-29  leading-dimension byte offset >> 4 (unused for swizzled K-major; 1)
//   bits 32-45  stride-dimension byte offset >> 4 (1024 B between 8-row atoms)
//   bits 46-48  fixed 0b001 (descriptor version for sm_100)
//   bits 49-51  base offset (0: atoms are 1024-byte aligned)
//   bit  52     LBO mode (0: relative)
//   bits 61-63  swizzle mode (2 = 128-byte swizzle)
// Stepping K inside the 128-byte atom is done by adding k*32 bytes to the start
// address (32 bytes = 16 f16/bf16 elements = 32 e4m3 elements = one MMA K-step).
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor for tcgen05.mma kind::f16 / kind::f8f6f4, dense, both
// operands K-major, fp32 accumulator.
//   bits  4-5   D format (1 = f32)
//   bits  7-9   A format (kind::f16: 0 f16, 1 bf16; kind::f8f6f4: 0 e4m3, 1 e5m2)
//   bits 10-12  B format (same encoding)
//   bit  15/16  A/B major (0 = K-major)
//   bits 17-22  N >> 3
//   bits 24-28  M >> 4
__host__ __device__ constexpr uint32_t idesc_f32acc(uint32_t a_fmt, uint32_t b_fmt, uint32_t M,
                                                    uint32_t N) {
  return (1u << 4) | (a_fmt << 7) | (b_fmt << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// ---------------------------------------------------------------------------------
// tcgen05: MMA + commit
// ---------------------------------------------------------------------------------
// kind: 0 = kind::f16 (f16/bf16 operands, K=16 per instruction)
//       1 = kind::f8f6f4 (e4m3/e5m2 operands, K=32 per instruction)
template <int CG, int KIND>
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                     uint32_t accumulate) {
  if constexpr (CG == 1 && KIND == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  } else if constexpr (CG == 1 && KIND == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  } else if constexpr (CG == 2 && KIND == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  }
}

// Arrive once on `bar` when every tcgen05 async operation issued so far by this
// thread has completed. `bar` is a shared::cluster address (a local shared::cta
// address is valid too).
template <int CG>
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
  else
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// Pair form: one commit that arrives on the barrier at the same shared-memory
// offset in every CTA of `cta_mask` (bit r = cluster rank r): a completion signal
// inside this GPU's own CTA pair. It moves no data.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          bar),
      "h"(cta_mask)
      : "memory");
}

// ---------------------------------------------------------------------------------
// tcgen05: TMEM -> registers. Shape 32x32b: thread t of the warp reads TMEM lane
// (lane_base + t); .xN reads N consecutive 32-bit columns. A warp may only touch
// the 32-lane quarter selected by (warp id % 4).
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------------
// Cluster launch control (hardware work stealing for persistent kernels)
// ---------------------------------------------------------------------------------
// Ask the hardware to cancel a cluster of this grid that has not started yet. The
// 16-byte response is written to `resp` (shared::cta) and 16 transaction bytes are
// credited to `bar`.
__device__ __forceinline__ void clc_try_cancel(uint32_t resp, uint32_t bar) {
  asm volatile(
      "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];" ::"r"(
          resp),
      "r"(bar)
      : "memory");
}

// Decode a response: returns true and the first CTA id (x) of the cancelled
// cluster, or false when no cluster was left to cancel.
__device__ __forceinline__ bool clc_decode(uint32_t resp, uint32_t& first_ctaid_x) {
  uint32_t ok, x;
  asm volatile(
      "{\n\t.reg .b128 r;\n\t.reg .pred p;\n\t"
      "ld.shared.b128 r, [%2];\n\t"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, r;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t"
      "clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %1, r;\n\t}"
      : "=r"(ok), "=r"(x)
      : "r"(resp)
      : "memory");
  first_ctaid_x = x;
  return ok != 0;
}

// ---------------------------------------------------------------------------------
// numeric packing for the epilogue
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

}  // namespace b200
