// Thin inline-PTX layer for sm_100a: mbarriers, TMA (no multicast), tcgen05 (TMEM alloc, MMA,
// commit, TMEM load/store), UMMA descriptors and bounded waits.
//
// This layer replaces three reference subsystems:
//   * common/cpasync.cuh:6-89      cp.async 16-byte copies        -> TMA cp.async.bulk.tensor
//   * common/mpmcq.cuh:10-115      global-memory ring queues      -> mbarrier full/empty rings in smem
//   * CUTLASS Sm80 mma.sync tiles (common/pipe_gemm_bias_relu.cuh:39-53) -> tcgen05.mma into TMEM
//
// Every wait is bounded: on expiry it records an error code in the kernel's status word and raises
// the CTA-local abort flag, so a lost arrival never hangs the GPU (the reference spins without
// bound at common/mpmcq.cuh:83 and :104).
#pragma once

#include <cstdint>
#include <type_traits>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace gp {

// ------------------------------------------------------------------------------------------------
// Status codes written by kernels into the per-device status word (host reads them back).
// ------------------------------------------------------------------------------------------------
enum DeviceStatus : int {
  kDevOk = 0,
  kDevTimeoutProducer = 0x100,  // producer gave up waiting for a free ring slot
  kDevTimeoutMma = 0x200,       // MMA issuer gave up waiting for operands
  kDevTimeoutEpilogue = 0x300,  // epilogue gave up waiting for an accumulator
  kDevTimeoutWeights = 0x400,   // weight staging never completed
  kDevBadSmemAlign = 0x500,     // dynamic shared memory not 1024-byte aligned
  kDevBadIndex = 0x600,         // a gather / scatter index outside [0, n_nodes): row read as zeros
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool elect_lane0() { return (threadIdx.x & 31) == 0; }

// ------------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Programmatic dependent launch. launch_dependents lets the next grid of the stream be scheduled
// once every CTA of this grid has issued it (its CTAs then take SMs as this grid's CTAs exit and
// run their set-up); wait blocks until the previous grid of the stream has completed and its
// memory operations are visible. A kernel touches global memory only after its wait. Both are
// no-ops in a launch without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void pdl_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t"
      "}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Cluster-scope variants (CTA pairs): the arrivals come from the peer CTA.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t"
      "}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_test_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t"
      "}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Arrive on an mbarrier given by its shared::cluster address (possibly in the peer CTA).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}

// shared::cluster address of the variable at `smem_addr` in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}

// Non-blocking probe of a phase (no suspend).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t"
      "}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Shared context for bounded waits: where to report, how long to wait, and the CTA abort flag.
struct WaitCtx {
  int* status;                 // device status word (global memory)
  volatile int* abort_flag;    // CTA-local flag in shared memory
  uint64_t timeout_ns;         // per-wait budget
};

// Wait until the phase with the given parity of `bar` has completed. Returns false (after
// recording `code` in the status word and raising the abort flag) if the budget runs out or
// another role of this CTA already aborted.
template <bool kCluster = false>
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtx& w,
                                          int code) {
  auto probe = [&]() {
    return kCluster ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
  };
  if (probe()) return true;
  // the clock is first read after 64 unsuccessful probes, so a wait that ends soon pays no
  // %globaltimer read; the budget then runs from that first read
  uint64_t t0 = 0;
  uint32_t spins = 0;
  while (true) {
    if (probe()) return true;
    if ((++spins & 63u) == 0) {
      if (*w.abort_flag) return false;
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > w.timeout_ns) {
        atomicCAS(w.status, 0, code);
        *w.abort_flag = 1;
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Async-proxy fences and TMA (cp.async.bulk.tensor). No load here uses cluster multicast: every
// CTA fetches its own tiles.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 2-D tiled load global -> shared, completion signalled on `bar` as transaction bytes.
// c0 is the innermost (contiguous) coordinate in elements, c1 the row.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// Same, with an L2 cache-policy hint (used to keep weights resident in L2).
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const void* tmap, uint32_t bar,
                                                 int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// CTA-pair form: the completion is signalled on `cluster_bar`, which may be the pair leader's
// barrier (shared::cluster address); the data lands in this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* tmap, uint32_t cluster_bar,
                                                 int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(cluster_bar), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// Four rows r0..r3 (any order, any rows; out-of-range rows read zeros) of a 2-D tensor, one
// box-width of columns from c0, into four consecutive 128-byte rows at dst (tile::gather4; the
// tensor map's box is one row high). CTA-pair form: completion on the leader's barrier.
__device__ __forceinline__ void tma_gather4_pair(uint32_t dst, const void* tmap, uint32_t cluster_bar, int c0,
                                                 int r0, int r1, int r2, int r3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5, %6, %7}], [%2], %8;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(cluster_bar), "r"(c0), "r"(r0), "r"(r1), "r"(r2), "r"(r3),
      "l"(policy)
      : "memory");
}

// 3-D tiled loads for weight stages: the tensor map views a row-major [K, N] matrix as
// {64 columns, K rows, N / 64 column blocks} (block stride 128 bytes), so one request fetches
// several 64-column blocks of a row range, laid out block after block in shared memory. TMA cost
// is largely per request, so one request per stage instead of one per 64-column block.
__device__ __forceinline__ void tma_load_3d_hint(uint32_t dst, const void* tmap, uint32_t bar, int c0,
                                                 int c1, int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const void* tmap, uint32_t cluster_bar,
                                                 int c0, int c1, int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(cluster_bar), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2-D tiled store shared -> global (rows/cols outside the tensor are clipped by the hardware).
__device__ __forceinline__ void tma_store_2d(const void* tmap, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::
                   "l"(reinterpret_cast<uint64_t>(tmap)),
               "r"(src), "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads/stores, fences
// ------------------------------------------------------------------------------------------------
// Whole-warp collective. Writes the TMEM base address to shared memory at `dst_smem`.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// CTA-pair (cta_group::2) TMEM management: executed by the same warp in both CTAs of the pair.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]; A holds two 16-bit values per 32-bit TMEM column.
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// CTA-pair MMA (issued by the pair leader only): M = 256 rows, 128 from each CTA's A operand;
// each CTA supplies N/2 columns of B; each CTA's TMEM receives its 128 rows x N.
__device__ __forceinline__ void mma_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Pair commit: arrive once on the barrier at the same shared-memory offset in every CTA of
// `cta_mask` when all previously issued tcgen05 ops of this thread finish.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          bar),
      "h"(cta_mask)
      : "memory");
}

// Arrive (count one) on `bar` once all previously issued tcgen05 async ops of this thread finish.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 bits, 32 consecutive columns: thread t of the warp receives lane (base+t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 32 bits, 16 consecutive columns.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// 32 lanes x 32 bits, 8 consecutive columns.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}

// ------------------------------------------------------------------------------------------------
// UMMA descriptors
// ------------------------------------------------------------------------------------------------
// Shared-memory matrix descriptor, SWIZZLE_128B, sm_100 version field = 1.
//   K-major operand: 8-row x 128-byte swizzle atoms, atoms stacked along M/N every `sbo` bytes;
//                    `lbo` unused (encoded as 16 bytes).
//   MN-major operand: 64-element (128-byte) MN blocks every `lbo` bytes, 8-row K groups every
//                    `sbo` bytes.
__device__ __forceinline__ uint64_t make_sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                     uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version (Blackwell)
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
//   ab_bf16: operand format (0 = f16, 1 = bf16); b_mn_major: B stored N-contiguous.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N, int ab_bf16, int a_mn_major,
                                                      int b_mn_major) {
  return (1u << 4)                                   // D format: f32
         | (static_cast<uint32_t>(ab_bf16) << 7)     // A format
         | (static_cast<uint32_t>(ab_bf16) << 10)    // B format
         | (static_cast<uint32_t>(a_mn_major) << 15) // A major
         | (static_cast<uint32_t>(b_mn_major) << 16) // B major
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

// ------------------------------------------------------------------------------------------------
// 16-bit element helpers (f16 / bf16 chosen at compile time)
// ------------------------------------------------------------------------------------------------
template <typename T>
struct Elem;

template <>
struct Elem<__half> {
  static constexpr int kIsBf16 = 0;
  static constexpr uint32_t kOneLow = 0x3C00u;  // 1.0 in the low half, 0 in the high half
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
  __device__ __forceinline__ static uint32_t pack_relu(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.relu.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  // inverse of pack: (low half, high half)
  __device__ __forceinline__ static float2 unpack(uint32_t v) {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
  }
};

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kIsBf16 = 1;
  static constexpr uint32_t kOneLow = 0x3F80u;
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
  __device__ __forceinline__ static uint32_t pack_relu(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static float2 unpack(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
  }
};

// ------------------------------------------------------------------------------------------------
// Activations applied in the epilogue (all in fp32 on the accumulator).
// ------------------------------------------------------------------------------------------------
enum Act : int { kActNone = 0, kActRelu = 1, kActGeluTanh = 2, kActSilu = 3, kActSigmoid = 4 };

// GELU, tanh form 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3))) (Hendrycks & Gimpel), with the
// hardware tanh approximation (tanh.approx.f32, max relative error about 2^-11, below the 16-bit
// rounding of the stored activation).
__device__ __forceinline__ float gelu_tanh_fast(float v) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * v, v * v, v);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * v * (1.0f + t);
}

// The logistic function through the identity sigmoid(v) = (1 + tanh(v / 2)) / 2 with the
// hardware tanh approximation: one special-function op per value instead of an exponential and
// a reciprocal (the epilogues of the wide SiLU chains are bound by that unit). Its absolute error
// stays below about 2^-12: below the 16-bit rounding of v * sigmoid(v) relative to |v|.
__device__ __forceinline__ float tanh_fast(float u) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return t;
}

// Activation chosen at compile time.
template <int ACT>
__device__ __forceinline__ float act_t(float v) {
  if constexpr (ACT == kActRelu) return fmaxf(v, 0.0f);
  else if constexpr (ACT == kActGeluTanh) return gelu_tanh_fast(v);
  else if constexpr (ACT == kActSilu) {
    const float h = 0.5f * v;  // v sigmoid(v) = h + h tanh(h)
    return fmaf(h, tanh_fast(h), h);
  } else if constexpr (ACT == kActSigmoid) return fmaf(0.5f, tanh_fast(0.5f * v), 0.5f);
  else return v;
}

__device__ __forceinline__ float apply_act(int act, float v) {
  switch (act) {
    case kActRelu: return act_t<kActRelu>(v);
    case kActGeluTanh: return act_t<kActGeluTanh>(v);
    case kActSilu: return act_t<kActSilu>(v);
    case kActSigmoid: return act_t<kActSigmoid>(v);
    default: return v;
  }
}

// Calls f(std::integral_constant<int, A>{}) for the runtime activation id `act`, so per-element
// code is specialised once per call site instead of switching per element.
template <class F>
__device__ __forceinline__ void act_dispatch(int act, F&& f) {
  switch (act) {
    case kActRelu: f(std::integral_constant<int, kActRelu>{}); break;
    case kActGeluTanh: f(std::integral_constant<int, kActGeluTanh>{}); break;
    case kActSilu: f(std::integral_constant<int, kActSilu>{}); break;
    case kActSigmoid: f(std::integral_constant<int, kActSigmoid>{}); break;
    default: f(std::integral_constant<int, kActNone>{}); break;
  }
}

}  // namespace gp
