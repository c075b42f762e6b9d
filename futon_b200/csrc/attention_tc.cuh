// attention_tc.cuh — variable-length self-attention on the 5th-generation
// tensor cores (tcgen05), restating native/model.go:646-739 (attendHead,
// softmaxScaled) for every head and sequence of a micro-batch at once.
//
// Work unit: a window of ≤ 128 query rows. Sequences of ≤ 128 tokens are
// packed whole into windows, each at a 16-row-aligned offset of the window
// (loaded as 16-row boxes); a window's keys are its own rows, masked so a
// query sees only its own sequence. Because every sequence starts on a
// 16-key boundary, the P·V MMAs (K = 16 keys each) group its keys exactly as
// they would alone: a sequence's vector does not depend on what it is packed
// with. Longer sequences get one window per 128 queries whose keys are the
// whole sequence in 128-key blocks. One CTA takes one window and loops over
// every head and key block ("unit" = head × key block):
//
//   warp 4 (one thread)  TMA: q, k, v tiles (128 rows × hd) of the unit into
//                        a two-slot shared-memory ring
//   warp 5 (one thread)  tcgen05.mma: S = Q·Kᵀ (bf16, M = 128, N = keys
//                        rounded to 16) into TMEM; after the softmax, O += P·V
//                        (f16, V read MN-major straight from its row-major
//                        tile) and L += P·1 (row sums) into TMEM
//   warps 0-3            softmax, one thread per query row (TMEM lane): two
//                        passes over its S row (max, then exp2 in f16x2 of the
//                        scaled, shifted scores), P (f16) into a 128-byte-
//                        swizzled K-major shared tile; online-softmax
//                        rescaling of O and L between key blocks; the
//                        normalised O row of each head to global memory
//
// Probability precision matches the mma.sync kernel: exponents rounded to
// f16 before ex2.approx.f16x2, P and V in f16, f32 accumulation. Packed
// windows fold the sequence mask into S = Q·Kᵀ as an extra K = 16 step
// (exact zeros inside a sequence), so the softmax never tests key indices.
#pragma once

#include <cuda_fp16.h>

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

template <int HD>
struct AttnTcCfg {
  static constexpr int kRowBytes = HD * 2;
  static constexpr int kTileBytes = 128 * kRowBytes;       // one q, k or v tile
  static constexpr int kSlotBytes = 3 * kTileBytes;
  static constexpr int kSlots = 2;
  static constexpr int kPOffset = kSlots * kSlotBytes;     // multiple of 1024
  static constexpr int kPBytes = 2 * 128 * 128;            // two 64-key regions, 128 B rows
  static constexpr int kOnesOffset = kPOffset + kPBytes;
  static constexpr int kOnesBytes = 16 * 128;              // B operand of the row sums
  // Packed windows: the sequence mask as one more K = 16 step of S = Q·Kᵀ —
  // row r of the q side holds onehot(segment(r)), row k of the k side holds
  // −30000·(1 − onehot(segment(k))), both bf16 in 64-byte swizzled rows.
  static constexpr int kAugOffset = kOnesOffset + 2048;    // 1024-aligned
  static constexpr int kAugBytes = 2 * 128 * 64;
  static constexpr int kBarOffset = kAugOffset + kAugBytes;
  static constexpr int kBytes = kBarOffset + 128 + 1024;   // + barriers + alignment slack
  static constexpr uint32_t kTmemCols = 256;
  static constexpr uint32_t kColO = 128;                   // S: columns 0-127
  static constexpr uint32_t kColL = 128 + HD;
  static constexpr int kThreads = 192;
};

template <int HD>
constexpr int attn_tc_smem_bytes() { return AttnTcCfg<HD>::kBytes; }

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

// grid = number of windows, block = 192. qkv: [T, 3h] (bf16 q, k; f16 v)
// read through tm_qkv (box hd × 128, long-sequence windows) and tm_qkv16
// (box hd × 16, packed windows).
template <int HD, typename OutT>
__global__ void __launch_bounds__(192, HD == 32 ? 2 : 1)
    attn_tc_kernel(const __grid_constant__ AttnMaps maps, int hidden, int num_heads,
                   const AttnWindow* __restrict__ windows, const AttnSeg* __restrict__ segs,
                   float scale_log2, OutT* __restrict__ out, int ldo, int* __restrict__ err) {
  using C = AttnTcCfg<HD>;
  extern __shared__ uint8_t sm_raw[];
  const uint32_t sbase = (smem_u32(sm_raw) + 1023u) & ~1023u;
  const uint32_t sP = sbase + C::kPOffset;
  const uint32_t sOnes = sbase + C::kOnesOffset;
  const uint32_t sQa = sbase + C::kAugOffset, sKa = sQa + 128 * 64;
  const uint32_t bars = sbase + C::kBarOffset;
  const uint32_t full_b = bars;            // [2] TMA → MMA
  const uint32_t empty_b = bars + 16;      // [2] MMA → TMA
  const uint32_t sfull_b = bars + 32;      // S ready (MMA → softmax)
  const uint32_t sfree_b = bars + 40;      // S read (softmax → MMA)
  const uint32_t pfull_b = bars + 48;      // P written, O corrected (softmax → MMA)
  const uint32_t ofull_b = bars + 56;      // P·V done (MMA → softmax)
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const AttnWindow win = windows[blockIdx.x];
  const bool packed = win.nseg > 0;
  const int nkb = (win.nk + 127) / 128;    // key blocks per head
  const int units = num_heads * nkb;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int i = 0; i < 2; ++i) {
      mbar_init(full_b + 8 * i, 1);
      mbar_init(empty_b + 8 * i, 1);
    }
    mbar_init(sfull_b, 1);
    mbar_init(sfree_b, 4);
    mbar_init(pfull_b, 4);
    mbar_init(ofull_b, 1);
    fence_barrier_init();
    for (int n = 1; n <= 8; ++n) tma_prefetch_desc(&maps.m[n]);
  }
  // The row-sum operand: 16 rows × 128 bytes of f16 ones (layout-independent).
  for (int i = threadIdx.x; i < C::kOnesBytes / 16; i += blockDim.x)
    st_shared_v4(sOnes + 16 * i, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);

  // Softmax thread = query row r: its token (−1: padding row) and, for
  // packed windows, its segment's rows [klo, khi) and the mask rows.
  const int r = warp * 32 + lane;
  int tok = -1, klo = 0, khi = 0;
  if (warp < 4) {
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
      // q side: onehot(segment); k side: −30000 off the own segment (bf16
      // 0xC6EA = −29952), so S gains 0 inside a sequence and about −3e4
      // across sequences or on padding keys.
      uint32_t qa[8], ka[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t lo = (2 * i == sidx) ? 0x3F80u : 0u, hi = (2 * i + 1 == sidx) ? 0x3F80u : 0u;
        qa[i] = lo | (hi << 16);
        const uint32_t klo16 = (2 * i == sidx) ? 0u : 0xC6EAu;
        const uint32_t khi16 = (2 * i + 1 == sidx) ? 0u : 0xC6EAu;
        ka[i] = klo16 | (khi16 << 16);
      }
      const int sw = (r >> 1) & 3;  // 64-byte swizzle: 16-byte chunk c at c ^ sw
      st_shared_v4(sQa + r * 64 + ((0 ^ sw) << 4), qa[0], qa[1], qa[2], qa[3]);
      st_shared_v4(sQa + r * 64 + ((1 ^ sw) << 4), qa[4], qa[5], qa[6], qa[7]);
      st_shared_v4(sKa + r * 64 + ((0 ^ sw) << 4), ka[0], ka[1], ka[2], ka[3]);
      st_shared_v4(sKa + r * 64 + ((1 ^ sw) << 4), ka[4], ka[5], ka[6], ka[7]);
    }
  }
  fence_proxy_async_smem();
  if (warp == 5) {
    tmem_alloc(smem_u32(&tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      for (int u = 0; u < units; ++u) {
        const int head = u / nkb, j = u % nkb, slot = u & 1;
        if (u >= 2 && !mbar_wait_bounded(empty_b + 8 * slot, ((u >> 1) - 1) & 1, err,
                                         kDevTimeoutAttn, &abort_flag))
          break;
        const uint32_t fb = full_b + 8 * slot;
        const uint32_t dst = sbase + slot * C::kSlotBytes;
        const int xq = head * HD, xk = hidden + head * HD, xv = 2 * hidden + head * HD;
        if (!packed) {
          mbar_arrive_expect_tx(fb, C::kSlotBytes);
          tma_load_2d(dst, &maps.m[8], fb, xq, win.q0);
          tma_load_2d(dst + C::kTileBytes, &maps.m[8], fb, xk, win.k0 + 128 * j);
          tma_load_2d(dst + 2 * C::kTileBytes, &maps.m[8], fb, xv, win.k0 + 128 * j);
        } else {
          // Rows [0, nq) in 16-row boxes, each segment from its own tokens.
          mbar_arrive_expect_tx(fb, 3 * win.nq * C::kRowBytes);
          for (int sg = 0; sg < win.nseg; ++sg) {
            const AttnSeg sq = segs[win.seg0 + sg];
            const CUtensorMap* mp = &maps.m[(sq.len + 15) >> 4];
            const uint32_t o = (uint32_t)sq.row * C::kRowBytes;
            tma_load_2d(dst + o, mp, fb, xq, sq.t0);
            tma_load_2d(dst + C::kTileBytes + o, mp, fb, xk, sq.t0);
            tma_load_2d(dst + 2 * C::kTileBytes + o, mp, fb, xv, sq.t0);
          }
        }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      auto keys16 = [&](int j) { return (min(128, win.nk - 128 * j) + 15) & ~15; };
      auto issue_s = [&](int u) -> bool {
        const int slot = u & 1;
        if (!mbar_wait_bounded(full_b + 8 * slot, (u >> 1) & 1, err, kDevTimeoutAttn, &abort_flag))
          return false;
        tc_fence_after();
        const uint32_t q = sbase + slot * C::kSlotBytes, k = q + C::kTileBytes;
        const uint32_t n = (uint32_t)keys16(u % nkb);
        const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | (8u << 24);
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          mma_bf16(tmem, desc_rows<HD>(q) + 2 * ks, desc_rows<HD>(k) + 2 * ks, idesc,
                   ks ? 1u : 0u);
        if (packed) mma_bf16(tmem, desc_rows<32>(sQa), desc_rows<32>(sKa), idesc, 1u);
        mma_commit(sfull_b);
        return true;
      };
      constexpr uint32_t idesc_pv = (1u << 4) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) | (8u << 24);
      constexpr uint32_t idesc_l = (1u << 4) | (2u << 17) | (8u << 24);
      bool ok = units > 0 && issue_s(0);
      for (int u = 0; ok && u < units; ++u) {
        // S(u + 1) as soon as the softmax has read S(u).
        if (!mbar_wait_bounded(sfree_b, u & 1, err, kDevTimeoutAttn, &abort_flag)) break;
        if (u + 1 < units && !issue_s(u + 1)) break;
        if (!mbar_wait_bounded(pfull_b, u & 1, err, kDevTimeoutAttn, &abort_flag)) break;
        tc_fence_after();
        const int j = u % nkb, slot = u & 1;
        const uint32_t v = sbase + slot * C::kSlotBytes + 2 * C::kTileBytes;
        const int nks = keys16(j) / 16;
        for (int ks = 0; ks < nks; ++ks) {
          const uint64_t pd = smem_desc_k_sw128(sP + (ks >> 2) * 16384) + 2 * (ks & 3);
          const uint32_t acc = (j > 0 || ks > 0) ? 1u : 0u;
          mma_bf16(tmem + C::kColO, pd, desc_rows<HD>(v + ks * 16 * C::kRowBytes), idesc_pv, acc);
          mma_bf16(tmem + C::kColL, pd, smem_desc_k_sw128(sOnes) + 2 * (ks & 3), idesc_l, acc);
        }
        mma_commit(ofull_b);
        mma_commit(empty_b + 8 * slot);
      }
    }
  } else {
    // ---------------- softmax warps 0-3: thread = query row ----------------
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    const uint32_t prow = sP + (uint32_t)r * 128u;
    const int swz = r & 7;
    // 32-key chunks any row of this warp needs (packed windows: its rows'
    // segments; long windows: the whole block); other chunks of P are zero.
    int clo = tok >= 0 ? klo >> 5 : 4, chi = tok >= 0 ? (khi + 31) >> 5 : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      clo = min(clo, __shfl_xor_sync(0xffffffffu, clo, o));
      chi = max(chi, __shfl_xor_sync(0xffffffffu, chi, o));
    }
    float m_run = -INFINITY;
    bool ok = true;

    // Normalised O row of `head` to global memory.
    auto store_head = [&](int head) {
      uint32_t ov[HD];
#pragma unroll
      for (int c = 0; c < HD; c += 32) {
        uint32_t t[32];
        tmem_ld32(trow + C::kColO + c, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) ov[c + i] = t[i];
      }
      const float l = __uint_as_float(tmem_ld1(trow + C::kColL));
      tmem_ld_wait();
      if (tok >= 0) {
        const float inv = rcp_approx(l);  // l ≥ 1: the row maximum contributes 2^0
        OutT* dst = out + (size_t)tok * ldo + head * HD;
        float y[32];
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
#pragma unroll
          for (int i = 0; i < 32; ++i) y[i] = __uint_as_float(ov[c + i]) * inv;
          store32<OutT>(dst + c, y);
        }
      }
    };

    for (int u = 0; u < units && ok; ++u) {
      const int head = u / nkb, j = u % nkb;
      if (j == 0) m_run = -INFINITY;  // a new head
      const int nkeys = min(128, win.nk - 128 * j);
      const int nchunk = (((nkeys + 15) & ~15) + 31) / 32;  // chunks the P·V MMAs read
      const int c0 = packed ? clo : 0;
      const int c1 = packed ? chi : (nkeys + 31) >> 5;
      if (!mbar_wait_bounded(sfull_b, u & 1, err, kDevTimeoutAttn, &abort_flag)) { ok = false; break; }
      tc_fence_after();
      // The row's scores of the live chunks, one TMEM wait for all.
      uint32_t sv[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c >= c0 && c < c1) tmem_ld32(trow + 32 * c, sv[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sfree_b);
      // Long windows: keys past the sequence in the last block (the same for
      // every row) leave the softmax.
      if (nkeys & 31) {
        const int c = (nkeys - 1) >> 5;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          if (cc == c) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (32 * cc + i >= nkeys) sv[cc][i] = __float_as_uint(-INFINITY);
          }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c >= c0 && c < c1) {
#pragma unroll
          for (int i = 0; i < 32; i += 2)
            mx = fmax3(mx, __uint_as_float(sv[c][i]), __uint_as_float(sv[c][i + 1]));
        }
      const float m_new = fmaxf(m_run, mx);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;  // rows without keys: P = 0
      const float alpha = ex2_approx(((m_run == -INFINITY ? m_use : m_run) - m_use) * scale_log2);
      m_run = m_new;
      const float ms = m_use * scale_log2;
      const uint64_t sl2 = f2_pack(scale_log2, scale_log2), nms2 = f2_pack(-ms, -ms);
      if (u > 0) {
        // The previous unit's P·V has finished: P may be overwritten, and O
        // holds either a finished head (store it) or this head's running sum.
        if (!mbar_wait_bounded(ofull_b, (u - 1) & 1, err, kDevTimeoutAttn, &abort_flag)) { ok = false; break; }
        tc_fence_after();
        if (j == 0) {
          store_head(head - 1);
        } else if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < HD; c += 32) {
            uint32_t t[32];
            tmem_ld32(trow + C::kColO + c, t);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] = __float_as_uint(__uint_as_float(t[i]) * alpha);
            tmem_st32(trow + C::kColO + c, t);
          }
          const float l = __uint_as_float(tmem_ld1(trow + C::kColL));
          tmem_ld_wait();
          tmem_st1(trow + C::kColL, __float_as_uint(l * alpha));
          tmem_st_wait();
        }
      }
      // P = 2^(s·c − m·c) in f16 → the 128-byte-swizzled K-major tile
      // (keys 0-63 | 64-127); chunks no row of the warp needs are zero.
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c < nchunk) {
          const uint32_t base = prow + (uint32_t)(c >> 1) * 16384u;
          if (c >= c0 && c < c1) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int k = 8 * i + 2 * e;
                float a, b;
                f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[c][k]), __uint_as_float(sv[c][k + 1])),
                                 sl2, nms2),
                          a, b);
                w[e] = ex2_h2(a, b);
              }
              st_shared_v4(base + (uint32_t)((((c & 1) * 4 + i) ^ swz) << 4), w[0], w[1], w[2], w[3]);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              st_shared_v4(base + (uint32_t)((((c & 1) * 4 + i) ^ swz) << 4), 0u, 0u, 0u, 0u);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pfull_b);
    }
    if (ok && units > 0 &&
        mbar_wait_bounded(ofull_b, (units - 1) & 1, err, kDevTimeoutAttn, &abort_flag)) {
      tc_fence_after();
      store_head(num_heads - 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace futon
