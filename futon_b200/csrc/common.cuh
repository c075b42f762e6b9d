// common.cuh — shared device helpers for the futon B200 encoder kernels.
//
// Hand-written PTX wrappers for sm_100a: mbarriers with bounded waits, TMA
// tile loads (no multicast anywhere in this library: it runs one replica per
// GPU on up to 8 GPUs), and the tcgen05 tensor-core / tensor-memory
// instructions. Every wait has a time limit; on expiry the waiting thread
// records an error code in a device word that the host reads after the
// forward, and the kernel unwinds instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace futon {

// Device error codes written to the per-device error word.
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutTmaFull = 1,     // MMA warp waited too long for a TMA stage
  kDevTimeoutSmemEmpty = 2,   // producer waited too long for a free stage
  kDevTimeoutAccFull = 3,     // epilogue waited too long for an accumulator
  kDevTimeoutAccEmpty = 4,    // MMA warp waited too long for the epilogue
  kDevBadShape = 5,           // a kernel was launched with an unsupported shape
  kDevBadInput = 6,           // a token id outside [0, vocab) reached the device
  kDevTimeoutAttn = 7,        // attention waited too long for a TMA stage
  kDevTimeoutLnPeer = 8,      // LayerNorm epilogue waited too long for a peer CTA's sums
  kDevTimeoutSelfTest = 9,    // futon_cuda_selftest_wait_timeout's deliberately unmet wait
};

// Wall-clock limit for any single barrier wait (nanoseconds). A healthy
// wait lasts microseconds; one second means the pipeline is broken.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

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
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Returns false (and
// records `code` in *err) if it did not within kWaitLimitNs, or if another
// thread already raised the CTA abort flag.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int* err,
                                                  int code, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicCAS(err, 0, code);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// ----------------------------------------------------------------------------
// Thread-block clusters: distributed shared memory and remote mbarriers
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of `saddr` (a shared::cta address of this CTA)
// in the CTA with cluster rank `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ void st_cluster_f64x2(uint32_t caddr, double a, double b) {
  asm volatile("st.shared::cluster.v2.f64 [%0], {%1, %2};" ::"r"(caddr), "d"(a), "d"(b)
               : "memory");
}

// Asynchronous 16-byte store into another CTA's shared memory (both
// addresses shared::cluster): completes `bytes` of the transaction count of
// that CTA's mbarrier `cbar` once the data has landed, with no fence on the
// sending side (the receiver's acquire wait on the mbarrier orders it).
__device__ __forceinline__ void st_async_f64x2(uint32_t caddr, double a, double b, uint32_t cbar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f64 [%0], {%1, %2}, [%3];" ::"r"(
          caddr),
      "d"(a), "d"(b), "r"(cbar)
      : "memory");
}

// Arrive on an mbarrier of another CTA of the cluster, releasing this
// thread's earlier writes at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// mbar_wait_bounded for phases completed by other CTAs of the cluster.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint32_t bar, uint32_t parity, int* err,
                                                          int code, volatile int* abort_flag) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicCAS(err, 0, code);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Every thread of every CTA of the cluster; orders earlier shared-memory
// initialisation (mbarrier.init) before any remote access.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// ----------------------------------------------------------------------------
// Programmatic dependent launch. A kernel launched with programmatic stream
// serialization may start while the kernel before it in the stream is still
// running; pdl_wait returns once that kernel has completed and its memory
// operations are visible, so every kernel of the forward calls it before it
// reads or writes global memory that another kernel of the call touches
// (only set-up — shared memory, TMEM, barriers, weights, the call's
// metadata — comes before it), then pdl_trigger lets the next kernel start.
// Both do nothing for a kernel launched without the attribute.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ----------------------------------------------------------------------------
// TMA (tiled, no multicast)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tile load into CTA shared memory, completing `bar` with the byte count.
// x is the innermost (contiguous) coordinate in elements; callers keep
// x * elem_size a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// The same load issued by either CTA of a CTA pair (cluster ranks 2i, 2i + 1)
// that feeds one cta_group::2 MMA: the data lands in this CTA's shared memory
// and the byte count completes `cbar`, a shared::cluster address of an
// mbarrier in either CTA of the pair (the pair's leader, even rank, counts
// both CTAs' bytes). No multicast: each CTA fetches its own tile.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t cbar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cbar), "r"(x), "r"(y)
      : "memory");
}

// ----------------------------------------------------------------------------
// tcgen05: tensor memory and 5th-generation tensor-core MMA
// ----------------------------------------------------------------------------
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
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] · B[smem]ᵀ, kind::f16: f16 or bf16 operands (both the
// same, as idesc says), f32 accumulate. One thread issues.
__device__ __forceinline__ void mma_f16kind(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same with signed 8-bit operands and exact s32 accumulation (kind::i8).
__device__ __forceinline__ void mma_s8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every MMA previously issued by this thread is done.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// cta_group::2 forms, for kernels whose MMAs span a CTA pair. A kernel uses
// one cta_group throughout: allocation, MMA, commit and deallocation. The
// allocation and deallocation are issued by the same warp of both CTAs (the
// pair gets the same TMEM address, written to `dst_smem` in each CTA).
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

// D (+)= A·Bᵀ over a CTA pair, issued by the even CTA only: M = 256 rows, A's
// rows 0-127 and B's first N/2 rows in the issuing CTA's shared memory, A's
// rows 128-255 and B's other N/2 rows at the same addresses in its peer; D
// rows 0-127 land in the issuing CTA's TMEM, rows 128-255 in the peer's,
// every one of the N columns in both.
__device__ __forceinline__ void mma_f16kind_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the mbarrier at shared::cta address `bar` of every CTA in
// `cta_mask` (the pair) when the pair MMAs issued so far are done.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}

// Loads 32 consecutive f32/s32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle that TMA's CU_TENSOR_MAP_SWIZZLE_128B writes: rows of 128
// bytes, 8-row (1024-byte) swizzle atoms stacked along M/N. LBO is unused for
// this layout (encoded 1), SBO = 1024 bytes, descriptor version 1 (sm_100),
// layout type 2 = SWIZZLE_128B. Tile bases are 1024-byte aligned, so the
// base-offset field stays 0.
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);         // start address
  d |= (uint64_t)1u << 16;                          // leading byte offset (unused)
  d |= (uint64_t)(1024u >> 4) << 32;                // stride byte offset
  d |= (uint64_t)1u << 46;                          // version
  d |= (uint64_t)2u << 61;                          // SWIZZLE_128B
  return d;
}

// Instruction descriptor (kind::f16 / kind::i8): dense, K-major A and B,
// M = m (128, or 256 for a CTA pair), N = n.
//   c_format (bits 4-5):  1 = F32, 2 = S32
//   a/b_format (7-9, 10-12): kind::f16 0 = F16, 1 = BF16; kind::i8 1 = S8
//   n_dim (17-22) = N >> 3, m_dim (24-28) = M >> 4
__host__ __device__ constexpr uint32_t make_idesc(uint32_t c_format, uint32_t ab_format,
                                                  uint32_t m, uint32_t n) {
  return (c_format << 4) | (ab_format << 7) | (ab_format << 10) | ((n >> 3) << 17) |
         ((m >> 4) << 24);
}

// ----------------------------------------------------------------------------
// Warp helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace futon
