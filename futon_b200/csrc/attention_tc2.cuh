// attention_tc2.cuh — tcgen05 attention with two softmax warpgroups and
// separate q·k and v rings (opt-in, FUTON_CUDA_ATTN=tc2), restating
// native/model.go:646-739 (attendHead, softmaxScaled) for every head and
// sequence of a micro-batch.
//
// A CTA takes one window of ≤ 128 query rows (sequences of ≤ 128 tokens
// packed at 16-row-aligned offsets with the sequence mask folded into S as
// one more K = 16 MMA step, or 128 queries of a longer sequence with its
// keys in 128-key blocks); exponents rounded to f16 before ex2.approx.f16x2,
// P and V in f16, f32 accumulation in TMEM. What changes is the pipeline.
// A unit u is one key block of 64 qkv columns (one box, 128-byte rows,
// 128-byte swizzle): for head_dim 32 a head PAIR, whose two heads go to the
// two softmax groups; for head_dim 64 one head, units alternating between
// the groups (head pairs in order, each pair's key blocks interleaved, so a
// group meets its head's key blocks in order):
//
//   warp 8 (one thread)  TMA: q and k of unit u into a three-stage ring,
//                        v into a separate two-stage ring, so the next
//                        units' q·k tiles are in flight two units ahead and
//                        a v tile is released as soon as its P·V is done;
//   warp 9 (one thread)  MMA, TMEM owner (512 columns): a group's next S as
//                        soon as it has read its current one; P·V once P is
//                        written;
//   warps 0-3, 4-7       softmax groups e = 0, 1, thread = query row. Each
//                        group owns its S (128 TMEM columns), O (64: for
//                        head_dim 32 P·V runs over both heads' value columns
//                        and the group reads its own 32), row sums (16)
//                        and P tile (32 KB). A group reads S(u) and frees it
//                        at once, so S(u + 1) is computed while the group
//                        waits for P·V(u − 1) (which frees its P tile and
//                        settles O) and writes P(u); the other group's work
//                        fills this group's waits.
//
// For head_dim 32, q·kᵀ of head e reads its 32 columns at byte 64·e of each
// 128-byte row (the start-address advance inside a swizzle atom that the
// GEMM's K steps use).
// Every wait is bounded (kDevTimeoutAttn); before exit the producer waits
// (time-bounded) for its last copies and the MMA thread for its last MMAs.
#pragma once

#include <cuda_fp16.h>

#include <type_traits>

#include "attention.cuh"
#include "common.cuh"
#include "gemm_tc.cuh"
#include "mathf32.cuh"

namespace futon {

// A sequence placed in a packed window: tokens [t0, t0 + len) at window
// rows [row, row + len), row a multiple of 16.
struct AttnSeg {
  int t0, len, row;
};

// nseg = 0: query rows [q0, q0 + nq) of one long sequence whose keys are
// [k0, k0 + nk) (micro-batch-local token indices), nq ≤ 128.
// nseg > 0: segments [seg0, seg0 + nseg) packed into rows [0, nq), nq = nk =
// the rows they occupy rounded to 16 (≤ 128).
struct AttnWindow {
  int q0, nq;
  int k0, nk;
  int seg0, nseg;
};

struct AttnMaps {
  CUtensorMap m[9];  // m[n]: boxes of 16·n rows × hd columns
};

// Descriptor of a tile of 128 rows × HD 16-bit values as TMA writes it with
// the swizzle spanning one row (64 B for HD 32, 128 B for HD 64): 8-row
// atoms stacked at 8 · row bytes. Used K-major for q and k and MN-major
// (idesc bit 16) for v, whose one swizzle atom spans all HD columns.
template <int HD>
__device__ __forceinline__ uint64_t desc_rows(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1u << 16;                               // leading byte offset (unused)
  d |= (uint64_t)((8u * HD * 2u) >> 4) << 32;            // stride byte offset: 8 rows
  d |= (uint64_t)1u << 46;                               // version
  d |= (uint64_t)(HD == 32 ? 4u : 2u) << 61;             // SWIZZLE_64B / SWIZZLE_128B
  return d;
}

__device__ __forceinline__ uint32_t tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  return r;
}
__device__ __forceinline__ void tmem_st1(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v)
               : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// 2^lo, 2^hi as one f16x2 word (exponents rounded to f16 first).
__device__ __forceinline__ uint32_t ex2_h2(float lo, float hi) {
  uint32_t t, r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(t) : "f"(hi), "f"(lo));
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(t));
  return r;
}


struct AttnTc2Cfg {
  static constexpr int kRowBytes = 128;                    // two heads × 32 × 2 B
  static constexpr int kTileBytes = 128 * kRowBytes;       // one q, k or v tile (16 KB)
  static constexpr int kQkStages = 3, kVStages = 2;
  static constexpr int kQkOffset = 0;                      // [3] q tile, k tile
  static constexpr int kVOffset = kQkStages * 2 * kTileBytes;
  static constexpr int kPOffset = kVOffset + kVStages * kTileBytes;
  static constexpr int kPBytes = 2 * 128 * 128;            // per group: two 64-key regions
  static constexpr int kOnesOffset = kPOffset + 2 * kPBytes;
  static constexpr int kOnesBytes = 16 * 128;
  static constexpr int kAugOffset = kOnesOffset + 2048;    // 1024-aligned
  static constexpr int kAugBytes = 2 * 128 * 64;
  static constexpr int kBarOffset = kAugOffset + kAugBytes;
  static constexpr int kBarBytes = 256;
  static constexpr int kBytes = kBarOffset + kBarBytes + 1024;  // + alignment slack
  static constexpr uint32_t kTmemCols = 512;
  // TMEM columns of group e: S at 128·e, O at 256 + 64·e, row sums at 384 + 32·e.
  static constexpr uint32_t kColS = 0, kColO = 256, kColL = 384;
  static constexpr int kThreads = 320;
};

constexpr int attn_tc2_smem_bytes() { return AttnTc2Cfg::kBytes; }

// grid = number of windows, block = 320; HD = 32 or 64, num_heads even; qkv
// [T, 3h] (bf16 q, k; f16 v) through maps.m[n] (boxes of 16·n rows × 64
// columns).
template <int HD, typename OutT>
__global__ void __launch_bounds__(320, 1)
    attn_tc2_kernel(const __grid_constant__ AttnMaps maps, int hidden, int num_heads,
                    const AttnWindow* __restrict__ windows, const AttnSeg* __restrict__ segs,
                    float scale_log2, OutT* __restrict__ out, int ldo, int* __restrict__ err) {
  static_assert(HD == 32 || HD == 64, "head_dim 32 or 64");
  using C = AttnTc2Cfg;
  constexpr bool kPair = HD == 32;          // a unit = a head pair (both groups)
  // f16 outputs: q and k are f16 too (else bf16); the mask rows' 1 and
  // −29952 in that format.
  constexpr bool kQF16 = std::is_same<OutT, __half>::value;
  constexpr uint32_t kOne16 = kQF16 ? 0x3C00u : 0x3F80u;
  constexpr uint32_t kOff16 = kQF16 ? 0xF750u : 0xC6EAu;
  extern __shared__ uint8_t sm_raw[];
  const uint32_t sbase = (smem_u32(sm_raw) + 1023u) & ~1023u;
  const uint32_t sOnes = sbase + C::kOnesOffset;
  const uint32_t sQa = sbase + C::kAugOffset, sKa = sQa + 128 * 64;
  const uint32_t bars = sbase + C::kBarOffset;
  const uint32_t qkfull_b = bars;          // [3] q, k landed (TMA → MMA)
  const uint32_t qkempty_b = bars + 24;    // [3] both S of the unit done (MMA → TMA)
  const uint32_t vfull_b = bars + 48;      // [2] v landed
  const uint32_t vempty_b = bars + 64;     // [2] both P·V of the unit done
  const uint32_t sfull_b = bars + 80;      // [2] S(u, e) ready (MMA → group e)
  const uint32_t sfree_b = bars + 96;      // [2] group e has read S(u, e) (4 warps)
  const uint32_t pfull_b = bars + 112;     // [2] P(u, e) written, O settled (4 warps)
  const uint32_t ofull_b = bars + 128;     // [2] P·V(u, e) done (MMA → group e)
  const uint32_t drain_b = bars + 144;     // the MMA thread's last MMAs are done
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const AttnWindow win = windows[blockIdx.x];
  const bool packed = win.nseg > 0;
  const int nkb = (win.nk + 127) / 128;     // key blocks per head
  const int units = (kPair ? num_heads / 2 : num_heads) * nkb;
  // Unit u's 64-column block and key block.
  auto unit_col = [&](int u) {
    return kPair ? (u / nkb) * 64 : (2 * (u / (2 * nkb)) + (u & 1)) * 64;
  };
  auto unit_kb = [&](int u) { return kPair ? u % nkb : (u % (2 * nkb)) >> 1; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int i = 0; i < C::kQkStages; ++i) {
      mbar_init(qkfull_b + 8 * i, 1);
      mbar_init(qkempty_b + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(vfull_b + 8 * i, 1);
      mbar_init(vempty_b + 8 * i, 1);
      mbar_init(sfull_b + 8 * i, 1);
      mbar_init(sfree_b + 8 * i, 4);
      mbar_init(pfull_b + 8 * i, 4);
      mbar_init(ofull_b + 8 * i, 1);
    }
    mbar_init(drain_b, 1);
    fence_barrier_init();
    for (int n = 1; n <= 8; ++n) tma_prefetch_desc(&maps.m[n]);
  }
  for (int i = threadIdx.x; i < C::kOnesBytes / 16; i += blockDim.x)
    st_shared_v4(sOnes + 16 * i, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);

  // Softmax thread: query row r of the window (both groups cover rows
  // 0-127); its token (−1: padding row) and its keys [klo, khi).
  const int grp = warp >> 2;               // 0, 1 for warps 0-7
  const int r = (warp & 3) * 32 + lane;
  int tok = -1, klo = 0, khi = 0;
  if (warp < 8) {
    int sidx = -1;
    if (!packed) {
      if (r < win.nq) {
        tok = win.q0 + r;
        khi = win.nk;
      }
    } else {
      for (int sg = 0; sg < win.nseg; ++sg) {
        const AttnSeg sq = segs[win.seg0 + sg];
        if (r >= sq.row && r < sq.row + sq.len) {
          tok = sq.t0 + (r - sq.row);
          klo = sq.row;
          khi = sq.row + sq.len;
          sidx = sg;
        }
      }
      if (grp == 0) {
        // Mask rows: q side onehot(segment), k side
        // −29952 off the own segment.
        uint32_t qa[8], ka[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t lo = (2 * i == sidx) ? kOne16 : 0u, hi = (2 * i + 1 == sidx) ? kOne16 : 0u;
          qa[i] = lo | (hi << 16);
          const uint32_t klo16 = (2 * i == sidx) ? 0u : kOff16;
          const uint32_t khi16 = (2 * i + 1 == sidx) ? 0u : kOff16;
          ka[i] = klo16 | (khi16 << 16);
        }
        const int sw = (r >> 1) & 3;
        st_shared_v4(sQa + r * 64 + ((0 ^ sw) << 4), qa[0], qa[1], qa[2], qa[3]);
        st_shared_v4(sQa + r * 64 + ((1 ^ sw) << 4), qa[4], qa[5], qa[6], qa[7]);
        st_shared_v4(sKa + r * 64 + ((0 ^ sw) << 4), ka[0], ka[1], ka[2], ka[3]);
        st_shared_v4(sKa + r * 64 + ((1 ^ sw) << 4), ka[4], ka[5], ka[6], ka[7]);
      }
    }
  }
  fence_proxy_async_smem();
  if (warp == 9) {
    tmem_alloc(smem_u32(&tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 8) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      // Loads rows [0, nq) of column block x into dst: one 128-row box for
      // a long window (rows from `row0`), one 16·n-row box per packed segment.
      auto load_rows = [&](uint32_t dst, uint32_t bar, int x, int row0) {
        if (!packed) {
          tma_load_2d(dst, &maps.m[8], bar, x, row0);
        } else {
          for (int sg = 0; sg < win.nseg; ++sg) {
            const AttnSeg sq = segs[win.seg0 + sg];
            tma_load_2d(dst + (uint32_t)sq.row * C::kRowBytes, &maps.m[(sq.len + 15) >> 4], bar, x,
                        sq.t0);
          }
        }
      };
      const uint32_t tile_tx = packed ? (uint32_t)win.nq * C::kRowBytes : (uint32_t)C::kTileBytes;
      int qk_issued = 0, v_issued = 0;
      auto issue_qk = [&](int u) -> bool {
        const int slot = u % C::kQkStages;
        if (u >= C::kQkStages &&
            !mbar_wait_bounded(qkempty_b + 8 * slot, (uint32_t)(u / C::kQkStages - 1) & 1u, err,
                               kDevTimeoutAttn, &abort_flag))
          return false;
        const int col = unit_col(u), j = unit_kb(u);
        const uint32_t fb = qkfull_b + 8 * slot;
        const uint32_t dst = sbase + C::kQkOffset + (uint32_t)slot * 2u * C::kTileBytes;
        mbar_arrive_expect_tx(fb, 2 * tile_tx);
        load_rows(dst, fb, col, win.q0);
        load_rows(dst + C::kTileBytes, fb, hidden + col, win.k0 + 128 * j);
        ++qk_issued;
        return true;
      };
      auto issue_v = [&](int u) -> bool {
        const int slot = u & 1;
        if (u >= 2 && !mbar_wait_bounded(vempty_b + 8 * slot, (uint32_t)((u >> 1) - 1) & 1u, err,
                                         kDevTimeoutAttn, &abort_flag))
          return false;
        const int col = unit_col(u), j = unit_kb(u);
        const uint32_t fb = vfull_b + 8 * slot;
        mbar_arrive_expect_tx(fb, tile_tx);
        load_rows(sbase + C::kVOffset + (uint32_t)slot * C::kTileBytes, fb, 2 * hidden + col,
                  win.k0 + 128 * j);
        ++v_issued;
        return true;
      };
      // q·k two units ahead of v: QK(0), QK(1), QK(2), V(0), QK(3), V(1), …
      // (QK(u + 2) needs only the S of unit u − 1 to be done, V(u) the P·V
      // of unit u − 2).
      bool ok = true;
      for (int u = 0; ok && u < units && u < 2; ++u) ok = issue_qk(u);
      for (int u = 0; ok && u < units; ++u) {
        if (u + 2 < units) ok = issue_qk(u + 2);
        if (ok) ok = issue_v(u);
      }
      // Drain (time-bounded, also after an abort): this thread's last copies
      // land before the CTA can exit.
      for (int u = qk_issued - 1; u >= 0 && u >= qk_issued - C::kQkStages; --u) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(qkfull_b + 8 * (u % C::kQkStages), (uint32_t)(u / C::kQkStages) & 1u))
          if (globaltimer_ns() - t0 > kWaitLimitNs) break;
      }
      for (int u = v_issued - 1; u >= 0 && u >= v_issued - 2; --u) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(vfull_b + 8 * (u & 1), (uint32_t)(u >> 1) & 1u))
          if (globaltimer_ns() - t0 > kWaitLimitNs) break;
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      auto keys16 = [&](int j) { return (min(128, win.nk - 128 * j) + 15) & ~15; };
      // S of unit u for group e = q · kᵀ (+ the mask step) into the group's S
      // columns; head_dim 32: head e's columns start 64 bytes into each row.
      auto issue_s = [&](int u, int e) {
        const uint32_t q = sbase + C::kQkOffset + (uint32_t)(u % C::kQkStages) * 2u * C::kTileBytes;
        const uint32_t k = q + C::kTileBytes;
        const uint32_t n = (uint32_t)keys16(unit_kb(u));
        const uint32_t ab = kQF16 ? 0u : 1u;  // operand format: f16 0, bf16 1
        const uint32_t idesc = (1u << 4) | (ab << 7) | (ab << 10) | ((n >> 3) << 17) | (8u << 24);
        const uint32_t d = tmem + C::kColS + 128u * (uint32_t)e;
        const uint64_t hoff = kPair ? 4u * (uint32_t)e : 0u;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          mma_f16kind(d, smem_desc_k_sw128(q) + hoff + 2 * ks, smem_desc_k_sw128(k) + hoff + 2 * ks,
                   idesc, ks ? 1u : 0u);
        if (packed) mma_f16kind(d, desc_rows<32>(sQa), desc_rows<32>(sKa), idesc, 1u);
        mma_commit(sfull_b + 8 * e);
      };
      constexpr uint32_t idesc_pv = (1u << 4) | (1u << 16) | ((uint32_t)(64 >> 3) << 17) | (8u << 24);
      constexpr uint32_t idesc_l = (1u << 4) | (2u << 17) | (8u << 24);
      // P·V of unit u for group e into the group's O and row-sum columns.
      auto issue_pv = [&](int u, int e) {
        const int j = unit_kb(u);
        const uint32_t v = sbase + C::kVOffset + (uint32_t)(u & 1) * C::kTileBytes;
        const uint32_t sp = sbase + C::kPOffset + (uint32_t)e * C::kPBytes;
        const int nks = keys16(j) / 16;
        for (int ks = 0; ks < nks; ++ks) {
          const uint64_t pd = smem_desc_k_sw128(sp + (ks >> 2) * 16384) + 2 * (ks & 3);
          const uint32_t acc = (j > 0 || ks > 0) ? 1u : 0u;
          mma_f16kind(tmem + C::kColO + 64u * (uint32_t)e, pd,
                   desc_rows<64>(v + ks * 16 * C::kRowBytes), idesc_pv, acc);
          mma_f16kind(tmem + C::kColL + 32u * (uint32_t)e, pd,
                   smem_desc_k_sw128(sOnes) + 2 * (ks & 3), idesc_l, acc);
        }
        mma_commit(ofull_b + 8 * e);
      };
      bool ok = units > 0;
      if constexpr (kPair) {
        if (ok) ok = mbar_wait_bounded(qkfull_b, 0u, err, kDevTimeoutAttn, &abort_flag);
        if (ok) {
          tc_fence_after();
          issue_s(0, 0);
          issue_s(0, 1);
          mma_commit(qkempty_b);
        }
      } else {
        // Units 0 and 1 start the two groups.
        for (int u = 0; ok && u < 2 && u < units; ++u) {
          ok = mbar_wait_bounded(qkfull_b + 8 * u, 0u, err, kDevTimeoutAttn, &abort_flag);
          if (ok) {
            tc_fence_after();
            issue_s(u, u & 1);
            mma_commit(qkempty_b + 8 * u);
          }
        }
      }
      for (int u = 0; ok && !kPair && u < units; ++u) {
        // Unit u belongs to group e = u mod 2 as its i-th; the group's next
        // unit is u + 2.
        const int e = u & 1, i = u >> 1;
        if (u + 2 < units) {
          const int w = u + 2, qs = w % C::kQkStages;
          if (!mbar_wait_bounded(qkfull_b + 8 * qs, (uint32_t)(w / C::kQkStages) & 1u, err,
                                 kDevTimeoutAttn, &abort_flag) ||
              !mbar_wait_bounded(sfree_b + 8 * e, (uint32_t)i & 1u, err, kDevTimeoutAttn,
                                 &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(w, e);
          mma_commit(qkempty_b + 8 * qs);
        }
        if (!mbar_wait_bounded(vfull_b + 8 * (u & 1), (uint32_t)(u >> 1) & 1u, err, kDevTimeoutAttn,
                               &abort_flag) ||
            !mbar_wait_bounded(pfull_b + 8 * e, (uint32_t)i & 1u, err, kDevTimeoutAttn,
                               &abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv(u, e);
        mma_commit(vempty_b + 8 * (u & 1));
      }
      for (int u = 0; ok && kPair && u < units; ++u) {
        // S(u + 1, ·) as soon as its q·k tiles are in and each group has read S(u).
        if (u + 1 < units) {
          const int nu = u + 1, qs = nu % C::kQkStages;
          if (!mbar_wait_bounded(qkfull_b + 8 * qs, (uint32_t)(nu / C::kQkStages) & 1u, err,
                                 kDevTimeoutAttn, &abort_flag))
            break;
          for (int e = 0; e < 2 && ok; ++e) {
            if (!mbar_wait_bounded(sfree_b + 8 * e, (uint32_t)u & 1u, err, kDevTimeoutAttn,
                                   &abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(nu, e);
          }
          if (!ok) break;
          mma_commit(qkempty_b + 8 * qs);
        }
        // P·V(u, ·) once its v tile is in and each group has written P(u).
        const int vs = u & 1;
        if (!mbar_wait_bounded(vfull_b + 8 * vs, (uint32_t)(u >> 1) & 1u, err, kDevTimeoutAttn,
                               &abort_flag))
          break;
        for (int e = 0; e < 2 && ok; ++e) {
          if (!mbar_wait_bounded(pfull_b + 8 * e, (uint32_t)u & 1u, err, kDevTimeoutAttn,
                                 &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(u, e);
        }
        if (!ok) break;
        mma_commit(vempty_b + 8 * vs);
      }
      // Drain (time-bounded): every MMA issued above completes before TMEM
      // is freed.
      mma_commit(drain_b);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain_b, 0u))
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
  } else {
    // ---------------- softmax groups: warps 0-3 (e = 0), 4-7 (e = 1) ----------------
    const int e = grp;
    const uint32_t lanes = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t srow = tmem + lanes + C::kColS + 128u * (uint32_t)e;
    // This group's O columns: head_dim 32 its head's 32 of the pair's 64.
    constexpr int kOCols = kPair ? 32 : 64;
    const uint32_t orow = tmem + lanes + C::kColO + 64u * (uint32_t)e + (kPair ? 32u * (uint32_t)e : 0u);
    const uint32_t lrow = tmem + lanes + C::kColL + 32u * (uint32_t)e;
    const uint32_t prow = sbase + C::kPOffset + (uint32_t)e * C::kPBytes + (uint32_t)r * 128u;
    const int swz = r & 7;
    int clo = tok >= 0 ? klo >> 5 : 4, chi = tok >= 0 ? (khi + 31) >> 5 : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      clo = min(clo, __shfl_xor_sync(0xffffffffu, clo, o));
      chi = max(chi, __shfl_xor_sync(0xffffffffu, chi, o));
    }
    float m_run = -INFINITY;
    bool ok = true;

    // The head of unit u (this group's).
    auto head_of = [&](int u) { return kPair ? 2 * (u / nkb) + e : unit_col(u) / 64; };
    // Normalised O row of head `head` to global memory.
    auto store_head = [&](int head) {
      const float l = __uint_as_float(tmem_ld1(lrow));
      tmem_ld_wait();
      const float inv = rcp_approx(l);  // l ≥ 1: the row maximum contributes 2^0
#pragma unroll
      for (int c = 0; c < kOCols; c += 32) {
        uint32_t t[32];
        tmem_ld32(orow + c, t);
        tmem_ld_wait();
        if (tok >= 0) {
          float y[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) y[i] = __uint_as_float(t[i]) * inv;
          store32<OutT>(out + (size_t)tok * ldo + head * HD + c, y);
        }
      }
    };

    // This group's units: every unit (head pairs) or every other one.
    const int ustep = kPair ? 1 : 2;
    const int mine = kPair ? units : units / 2;
    for (int i = 0, u = kPair ? 0 : e; i < mine && ok; ++i, u += ustep) {
      const int j = unit_kb(u);
      if (j == 0) m_run = -INFINITY;  // a new head
      const int nkeys = min(128, win.nk - 128 * j);
      const int nchunk = (((nkeys + 15) & ~15) + 31) / 32;  // chunks the P·V MMAs read
      const int c0 = packed ? clo : 0;
      const int c1 = packed ? chi : (nkeys + 31) >> 5;
      if (!mbar_wait_bounded(sfull_b + 8 * e, (uint32_t)i & 1u, err, kDevTimeoutAttn,
                             &abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c >= c0 && c < c1) tmem_ld32(srow + 32 * c, sv[c]);
      tmem_ld_wait();
      // S(u) is in registers: the MMA thread may write S(u + 1).
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sfree_b + 8 * e);
      if (nkeys & 31) {
        const int c = (nkeys - 1) >> 5;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          if (cc == c) {
#pragma unroll
            for (int x = 0; x < 32; ++x)
              if (32 * cc + x >= nkeys) sv[cc][x] = __float_as_uint(-INFINITY);
          }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c >= c0 && c < c1) {
#pragma unroll
          for (int x = 0; x < 32; x += 2)
            mx = fmax3(mx, __uint_as_float(sv[c][x]), __uint_as_float(sv[c][x + 1]));
        }
      const float m_new = fmaxf(m_run, mx);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;  // rows without keys: P = 0
      const float alpha = ex2_approx(((m_run == -INFINITY ? m_use : m_run) - m_use) * scale_log2);
      m_run = m_new;
      const float ms = m_use * scale_log2;
      const uint64_t sl2 = f2_pack(scale_log2, scale_log2), nms2 = f2_pack(-ms, -ms);
      if (i > 0) {
        // The group's previous P·V has finished: P_e may be overwritten, and
        // O_e holds either a finished head or this head's running sum (dealt
        // with after the P write, once S is out of registers).
        if (!mbar_wait_bounded(ofull_b + 8 * e, (uint32_t)(i - 1) & 1u, err, kDevTimeoutAttn,
                               &abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      // P(u) = 2^(s·c − m·c) in f16 → this group's 128-byte-swizzled K-major
      // tile (keys 0-63 | 64-127); chunks no row of the warp needs are zero.
      // (Forming P before the wait above would hide P·V(u − 1) behind the
      // exponentials, but S and P together need more than the 168 registers
      // a 10-warp CTA leaves each thread.)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c < nchunk) {
          const uint32_t base = prow + (uint32_t)(c >> 1) * 16384u;
          if (c >= c0 && c < c1) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {  // 16-byte granule g of the chunk's 64 bytes
              uint32_t w[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int k = 8 * g + 2 * q;
                float a, b;
                f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[c][k]), __uint_as_float(sv[c][k + 1])),
                                 sl2, nms2),
                          a, b);
                w[q] = ex2_h2(a, b);
              }
              st_shared_v4(base + (uint32_t)((((c & 1) * 4 + g) ^ swz) << 4), w[0], w[1], w[2], w[3]);
            }
          } else {
#pragma unroll
            for (int g = 0; g < 4; ++g)
              st_shared_v4(base + (uint32_t)((((c & 1) * 4 + g) ^ swz) << 4), 0u, 0u, 0u, 0u);
          }
        }
      }
      if (i > 0) {
        if (j == 0) {
          store_head(head_of(u - ustep));
        } else if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < kOCols; c += 32) {
            uint32_t t[32];
            tmem_ld32(orow + c, t);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 32; ++q) t[q] = __float_as_uint(__uint_as_float(t[q]) * alpha);
            tmem_st32(orow + c, t);
          }
          const float l = __uint_as_float(tmem_ld1(lrow));
          tmem_ld_wait();
          tmem_st1(lrow, __float_as_uint(l * alpha));
          tmem_st_wait();
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pfull_b + 8 * e);
    }
    if (ok && mine > 0 &&
        mbar_wait_bounded(ofull_b + 8 * e, (uint32_t)(mine - 1) & 1u, err, kDevTimeoutAttn,
                          &abort_flag)) {
      tc_fence_after();
      store_head(head_of(kPair ? units - 1 : units - 2 + e));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace futon
