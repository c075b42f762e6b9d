// attention.cuh — variable-length multi-head self-attention over packed
// sequences (cu_seqlens), restating native/model.go:646-739 (attendHead,
// rotateHalf, softmaxScaled) for every head and sequence at once.
//
// The reference materialises a seq×padSeq(seq) score matrix per head; here
// scores never leave the SM. Queries, keys and values are read straight from
// the fused [T, 3h] qkv buffer (q columns head·hd, k columns h + head·hd,
// v columns 2h + head·hd, model.go:660-662). q and k arrive rotated: NeoX
// RoPE (model.go:674-685) runs in the qkv GEMM epilogue, on the f32
// accumulator.
//
// Kernels:
//   attn_heads_kernel  one 64-query tile of one sequence per CTA, all heads
//                      in turn (two per step for head_dim 32), 64-key tiles
//                      staged by TMA in a two-slot mbarrier ring, m16n8k16
//                      tensor-core MMAs with f32 accumulation
//                      (Q·Kᵀ in bf16, P·V in f16 — v is stored as f16) and
//                      online softmax (head_dim 32 or 64); also the CLS-only
//                      last layer (model.go:403-410).
//   attn_flash_split_kernel  int8 path: 64 queries × one head per CTA over
//                      f32 qkv, every operand split into bf16 hi + lo parts.
//   attn_rowq_kernel   one warp per (query, head): lanes split the keys,
//                      f32 math, warp merge (head dims other than 32/64).
#pragma once

#include <cuda_fp16.h>

#include <type_traits>

#include "common.cuh"
#include "mathf32.cuh"

namespace futon {

struct AttnTile {
  int seq;  // sequence index within the micro-batch
  int q0;   // first query position of the tile
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4],
                                          const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// D = A·B (no accumulator input).
__device__ __forceinline__ void mma_16816_z(float (&d)[4], const uint32_t (&a)[4],
                                            const uint32_t (&b)[2]) {
  const float z = 0.f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "f"(z));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

template <typename T> __device__ __forceinline__ void store2(T* dst, float a, float b);
template <> __device__ __forceinline__ void store2<float>(float* dst, float a, float b) {
  *reinterpret_cast<float2*>(dst) = make_float2(a, b);
}
template <> __device__ __forceinline__ void store2<__nv_bfloat16>(__nv_bfloat16* dst, float a,
                                                                  float b) {
  *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(a, b);
}
template <> __device__ __forceinline__ void store2<__half>(__half* dst, float a, float b) {
  uint32_t w;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(w) : "f"(b), "f"(a));
  *reinterpret_cast<uint32_t*>(dst) = w;
}

// ---------------------------------------------------------------------------
// Split-precision variant for the int8 path. The int8 path quantises the
// attention output per row, and int8 rounding boundaries amplify any input
// perturbation, so its attention must track float32 closely: q, k, v (f32)
// and the probabilities are each split into bf16 hi + lo parts and every
// product runs as hi·hi + hi·lo + lo·hi (relative error ≈ 2^-16).
// ---------------------------------------------------------------------------
template <int HD, bool ROPE>
__device__ __forceinline__ void stage_rows_split(__nv_bfloat16* dhi, __nv_bfloat16* dlo, int lds,
                                                 const float* src, int ld, int r0, int L,
                                                 const float* rcos, const float* rsin) {
  constexpr int kRows = 64, kHalf = HD / 2;
  constexpr int kItems = ROPE ? kRows * kHalf : kRows * HD;
  for (int w = threadIdx.x; w < kItems; w += blockDim.x) {
    if constexpr (ROPE) {
      const int r = w / kHalf, i = w % kHalf, pos = r0 + r;
      float y1 = 0.f, y2 = 0.f;
      if (pos < L) {
        const float x1 = src[(size_t)pos * ld + i], x2 = src[(size_t)pos * ld + i + kHalf];
        const float c = rcos[(size_t)pos * kHalf + i], sn = rsin[(size_t)pos * kHalf + i];
        y1 = x1 * c - x2 * sn;
        y2 = x2 * c + x1 * sn;
      }
      const __nv_bfloat16 h1 = __float2bfloat16_rn(y1), h2 = __float2bfloat16_rn(y2);
      dhi[r * lds + i] = h1;
      dlo[r * lds + i] = __float2bfloat16_rn(y1 - __bfloat162float(h1));
      dhi[r * lds + i + kHalf] = h2;
      dlo[r * lds + i + kHalf] = __float2bfloat16_rn(y2 - __bfloat162float(h2));
    } else {
      const int r = w / HD, i = w % HD, pos = r0 + r;
      const float y = pos < L ? src[(size_t)pos * ld + i] : 0.f;
      const __nv_bfloat16 hv = __float2bfloat16_rn(y);
      dhi[r * lds + i] = hv;
      dlo[r * lds + i] = __float2bfloat16_rn(y - __bfloat162float(hv));
    }
  }
}

// grid = (num_tiles, num_heads), block = 128, dynamic smem = 6 · 64 · (HD+8) bf16.
template <int HD, bool ROPE>
__global__ void __launch_bounds__(128)
    attn_flash_split_kernel(const float* __restrict__ qkv, int hidden,
                            const int* __restrict__ cu_seqlens, const AttnTile* __restrict__ tiles,
                            const float* __restrict__ rcos, const float* __restrict__ rsin,
                            float scale_log2, float* __restrict__ out, int ldo) {
  constexpr int kBK = 64, kLds = HD + 8, kTile = 64 * kLds;
  extern __shared__ __align__(16) __nv_bfloat16 sm[];
  __nv_bfloat16 *sQh = sm, *sQl = sm + kTile, *sKh = sm + 2 * kTile, *sKl = sm + 3 * kTile;
  __nv_bfloat16 *sVh = sm + 4 * kTile, *sVl = sm + 5 * kTile;

  const AttnTile tile = tiles[blockIdx.x];
  const int head = blockIdx.y;
  const int s0 = cu_seqlens[tile.seq];
  const int L = cu_seqlens[tile.seq + 1] - s0;
  const int ld = 3 * hidden;
  const float* qg = qkv + (size_t)s0 * ld + head * HD;
  const float* kg = qg + hidden;
  const float* vg = qg + 2 * hidden;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  stage_rows_split<HD, ROPE>(sQh, sQl, kLds, qg, ld, tile.q0, L, rcos, rsin);
  __syncthreads();
  uint32_t qh[HD / 16][4], ql[HD / 16][4];
#pragma unroll
  for (int kc = 0; kc < HD / 16; ++kc) {
    const int off = (warp * 16 + (lane & 15)) * kLds + kc * 16 + (lane >> 4) * 8;
    ldsm_x4(qh[kc], smem_u32(&sQh[off]));
    ldsm_x4(ql[kc], smem_u32(&sQl[off]));
  }
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  for (int kv0 = 0; kv0 < L; kv0 += kBK) {
    __syncthreads();
    stage_rows_split<HD, ROPE>(sKh, sKl, kLds, kg, ld, kv0, L, rcos, rsin);
    stage_rows_split<HD, false>(sVh, sVl, kLds, vg, ld, kv0, L, nullptr, nullptr);
    __syncthreads();
    float s[kBK / 8][4];
#pragma unroll
    for (int nb = 0; nb < kBK / 8; ++nb) {
      s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
#pragma unroll
      for (int kc = 0; kc < HD / 16; ++kc) {
        const int off = (nb * 8 + (lane & 7)) * kLds + kc * 16 + ((lane >> 3) & 1) * 8;
        uint32_t kh[2], kl[2];
        ldsm_x2(kh, smem_u32(&sKh[off]));
        ldsm_x2(kl, smem_u32(&sKl[off]));
        mma_16816(s[nb], ql[kc], kh);
        mma_16816(s[nb], qh[kc], kl);
        mma_16816(s[nb], qh[kc], kh);
      }
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < kBK / 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kv0 + nb * 8 + (lane & 3) * 2 + (e & 1);
        const float v = (key < L) ? s[nb][e] * scale_log2 : -INFINITY;
        s[nb][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float m_new = fmaxf(m_run[r], mx[r]);
      alpha[r] = (m_run[r] == -INFINITY) ? 0.f : exp2f(m_run[r] - m_new);
      m_run[r] = m_new;
      l_run[r] *= alpha[r];
    }
#pragma unroll
    for (int nb = 0; nb < kBK / 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(s[nb][e] - m_run[e >> 1]);
        s[nb][e] = p;
        l_run[e >> 1] += p;
      }
#pragma unroll
    for (int nd = 0; nd < HD / 8; ++nd) {
      o[nd][0] *= alpha[0]; o[nd][1] *= alpha[0];
      o[nd][2] *= alpha[1]; o[nd][3] *= alpha[1];
    }
#pragma unroll
    for (int kc = 0; kc < kBK / 16; ++kc) {
      float pv[8] = {s[2 * kc][0], s[2 * kc][1], s[2 * kc][2], s[2 * kc][3],
                     s[2 * kc + 1][0], s[2 * kc + 1][1], s[2 * kc + 1][2], s[2 * kc + 1][3]};
      float lo[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        lo[i] = pv[i] - __bfloat162float(__float2bfloat16_rn(pv[i]));
      uint32_t ph[4] = {pack_bf16(pv[0], pv[1]), pack_bf16(pv[2], pv[3]), pack_bf16(pv[4], pv[5]),
                        pack_bf16(pv[6], pv[7])};
      uint32_t pl[4] = {pack_bf16(lo[0], lo[1]), pack_bf16(lo[2], lo[3]), pack_bf16(lo[4], lo[5]),
                        pack_bf16(lo[6], lo[7])};
#pragma unroll
      for (int nd = 0; nd < HD / 8; ++nd) {
        const int off = (kc * 16 + (lane & 15)) * kLds + nd * 8;
        uint32_t vh[2], vl[2];
        ldsm_x2_t(vh, smem_u32(&sVh[off]));
        ldsm_x2_t(vl, smem_u32(&sVl[off]));
        mma_16816(o[nd], pl, vh);
        mma_16816(o[nd], ph, vl);
        mma_16816(o[nd], ph, vh);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  const float inv0 = 1.f / l_run[0], inv1 = 1.f / l_run[1];
  const int qr0 = tile.q0 + warp * 16 + (lane >> 2), qr1 = qr0 + 8;
#pragma unroll
  for (int nd = 0; nd < HD / 8; ++nd) {
    const int col = head * HD + nd * 8 + (lane & 3) * 2;
    if (qr0 < L) store2<float>(out + (size_t)(s0 + qr0) * ldo + col, o[nd][0] * inv0, o[nd][1] * inv0);
    if (qr1 < L) store2<float>(out + (size_t)(s0 + qr1) * ldo + col, o[nd][2] * inv1, o[nd][3] * inv1);
  }
}

// ---------------------------------------------------------------------------
// cp.async staging (the int8 path's split-precision kernel).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait1() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}

// 64 rows × HD bf16 of one head into shared memory (row stride HD + 8);
// rows at or past `lim` are zero-filled without reading.
template <int HD>
__device__ __forceinline__ void stage_async(__nv_bfloat16* dst, const __nv_bfloat16* src, int ld,
                                            int r0, int lim) {
  constexpr int kChunks = HD / 8, kLds = HD + 8;
  for (int w = threadIdx.x; w < 64 * kChunks; w += blockDim.x) {
    const int r = w / kChunks, c = (w % kChunks) * 8;
    const bool ok = r0 + r < lim;
    cp_async16(smem_u32(dst + r * kLds + c), ok ? src + (size_t)(r0 + r) * ld + c : src, ok);
  }
}

// ---------------------------------------------------------------------------
// attn_heads_kernel staging. Per (head group, 64-key tile) step one thread
// loads q (first tile of a group), k and v as 64 × (NH·HD) tiles of the
// [T, 3h] qkv buffer with TMA into a kAttnRing-slot shared-memory ring; each
// slot's mbarrier completes when its bytes land, so the next step's loads
// overlap this step's tensor-core work. Tiles are dense with the TMA swizzle
// whose span is one row (64 B for 32 columns, 128 B for 64), which keeps
// every ldmatrix phase (8 rows × 16 B) free of bank conflicts.
// ---------------------------------------------------------------------------
constexpr int kAttnRing = 2;

template <int W>  // tile width in elements (head_dim × heads per step)
struct AttnSmem {
  static constexpr int kRowBytes = W * 2;
  static constexpr int kTileBytes = 64 * kRowBytes;
  static constexpr int kBarOffset = 3 * kAttnRing * kTileBytes;
  static constexpr int kBytes = kBarOffset + 64 + 1024;  // + barriers + alignment slack
};

// Heads per (key tile) step: two for head_dim 32 (one 64-column TMA box
// holds both, so every barrier, wait and load serves twice the work), else one.
__host__ __device__ constexpr int attn_heads_per_step(int hd, int num_heads) {
  return hd == 32 && num_heads % 2 == 0 ? 2 : 1;
}

template <int HD, int NH>
constexpr int attn_heads_smem_bytes() { return AttnSmem<HD * NH>::kBytes; }

// The swizzle's XOR term for a tile row of RB bytes (64-byte swizzle for
// 64-byte rows, 128-byte swizzle for 128-byte rows): 16-byte chunk c of row r
// sits at chunk c ^ attn_swz(r). Every fragment row used below is a
// lane-dependent row plus a multiple of 8, which leaves the term unchanged.
template <int RB>
__device__ __forceinline__ int attn_swz(int r) {
  return RB == 64 ? (r >> 1) & 3 : r & 7;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void mma_16816_f16(float (&d)[4], const uint32_t (&a)[4],
                                              const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// D = A·B (+ D unless ZERO_C), f16 operands.
template <bool ZERO_C>
__device__ __forceinline__ void mma_16816_f16c(float (&d)[4], const uint32_t (&a)[4],
                                               const uint32_t (&b)[2]) {
  if constexpr (ZERO_C) {
    const float z = 0.f;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "f"(z));
  } else {
    mma_16816_f16(d, a, b);
  }
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^lo, 2^hi as one f16x2 word (lo in the low half): the exponents are
// rounded to f16 (relative error of the power ≤ 2^-11·|t|·ln 2, so at most
// 2^-12 where the probability is above 1/2 and 2^-8 where it is below 2^-8)
// and the powers come back in f16 — the A operand of the P·V MMA as is.
__device__ __forceinline__ uint32_t ex2_f16x2(float lo, float hi) {
  uint32_t t, r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(t) : "f"(hi), "f"(lo));
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(t));
  return r;
}

// One (head, key tile) step of one warp over its 16 query rows: S = Q Kᵀ on
// the NBLK 8-key blocks that hold keys, masking (PARTIAL: keys ≥ nkeys in the
// last block), online softmax with the scale folded into the exponent, and
// O += P V with P and V in f16. The softmax denominators come out of the
// same MMAs: a ninth (fifth) B block of ones sums each row of P exactly as
// it is multiplied. FIRST: the head's first key tile (no rescale of O).
// Per-lane byte offsets of the ldmatrix rows of head e inside a swizzled
// 64-row tile of RB-byte rows (head e holds 16-byte chunks e·HD/8 onward):
// k_off[i] for key chunks 4i..4i+3 (x4: rows nb·8 + lane%8), v_off[i] for
// value columns 16i..16i+15 (x4.trans: rows kc·16 + lane%16).
template <int HD, int RB>
struct AttnLane {
  uint32_t k_off[HD / 32];
  uint32_t v_off[HD / 16];
  AttnLane() = default;
  __device__ __forceinline__ AttnLane(int lane, int e) {
    const int kr = lane & 7, vr = lane & 15, c0 = e * (HD / 8);
#pragma unroll
    for (int i = 0; i < HD / 32; ++i)
      k_off[i] = kr * RB + (((c0 + (lane >> 3) + 4 * i) ^ attn_swz<RB>(kr)) << 4);
#pragma unroll
    for (int i = 0; i < HD / 16; ++i)
      v_off[i] = vr * RB + (((c0 + (lane >> 4) + 2 * i) ^ attn_swz<RB>(vr)) << 4);
  }
};

// QF16: q and k are f16 (else bf16).
template <int HD, int RB, int NBLK, bool PARTIAL, bool FIRST, bool QF16>
__device__ __forceinline__ void attn_step(uint32_t kS, uint32_t vS, const AttnLane<HD, RB>& al,
                                          int lane, int nkeys, float scale_log2,
                                          const uint32_t (&qf)[HD / 16][4],
                                          float (&o)[HD / 8][4], float (&m_run)[2],
                                          float (&lsum)[4]) {
  float sc[NBLK][4];
#pragma unroll
  for (int nb = 0; nb < NBLK; ++nb) {
#pragma unroll
    for (int kc = 0; kc < HD / 16; kc += 2) {
      uint32_t kf[4];
      ldsm_x4(kf, kS + nb * 8 * RB + al.k_off[kc / 2]);
      const uint32_t k0[2] = {kf[0], kf[1]}, k1[2] = {kf[2], kf[3]};
      if constexpr (QF16) {
        if (kc == 0) mma_16816_f16c<true>(sc[nb], qf[kc], k0);
        else mma_16816_f16c<false>(sc[nb], qf[kc], k0);
        mma_16816_f16c<false>(sc[nb], qf[kc + 1], k1);
      } else {
        if (kc == 0) mma_16816_z(sc[nb], qf[kc], k0);
        else mma_16816(sc[nb], qf[kc], k0);
        mma_16816(sc[nb], qf[kc + 1], k1);
      }
    }
  }
  if constexpr (PARTIAL) {
    const int key0 = (NBLK - 1) * 8 + (lane & 3) * 2;
    if (key0 >= nkeys) { sc[NBLK - 1][0] = -INFINITY; sc[NBLK - 1][2] = -INFINITY; }
    if (key0 + 1 >= nkeys) { sc[NBLK - 1][1] = -INFINITY; sc[NBLK - 1][3] = -INFINITY; }
  }
  float mx0 = fmaxf(sc[0][0], sc[0][1]), mx1 = fmaxf(sc[0][2], sc[0][3]);
#pragma unroll
  for (int nb = 1; nb < NBLK; ++nb) {
    mx0 = fmax3(mx0, sc[nb][0], sc[nb][1]);
    mx1 = fmax3(mx1, sc[nb][2], sc[nb][3]);
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  if constexpr (FIRST) {
    m_run[0] = mx0;
    m_run[1] = mx1;
  } else {
    const float n0 = fmaxf(m_run[0], mx0), n1 = fmaxf(m_run[1], mx1);
    const float a0 = ex2_approx((m_run[0] - n0) * scale_log2);
    const float a1 = ex2_approx((m_run[1] - n1) * scale_log2);
    m_run[0] = n0;
    m_run[1] = n1;
    const uint64_t r0 = f2_pack(a0, a0), r1 = f2_pack(a1, a1);
#pragma unroll
    for (int nd = 0; nd < HD / 8; ++nd) {
      f2_unpack(f2_mul(f2_pack(o[nd][0], o[nd][1]), r0), o[nd][0], o[nd][1]);
      f2_unpack(f2_mul(f2_pack(o[nd][2], o[nd][3]), r1), o[nd][2], o[nd][3]);
    }
    f2_unpack(f2_mul(f2_pack(lsum[0], lsum[1]), r0), lsum[0], lsum[1]);
    f2_unpack(f2_mul(f2_pack(lsum[2], lsum[3]), r1), lsum[2], lsum[3]);
  }
  const float ms0 = m_run[0] * scale_log2, ms1 = m_run[1] * scale_log2;
  const uint64_t sl = f2_pack(scale_log2, scale_log2);
  const uint64_t nm0 = f2_pack(-ms0, -ms0), nm1 = f2_pack(-ms1, -ms1);
  uint32_t pw[NBLK][2];  // P as f16x2: [block][row half]
#pragma unroll
  for (int nb = 0; nb < NBLK; ++nb) {
    float t0, t1, t2, t3;
    f2_unpack(f2_fma(f2_pack(sc[nb][0], sc[nb][1]), sl, nm0), t0, t1);
    f2_unpack(f2_fma(f2_pack(sc[nb][2], sc[nb][3]), sl, nm1), t2, t3);
    pw[nb][0] = ex2_f16x2(t0, t1);
    pw[nb][1] = ex2_f16x2(t2, t3);
  }
  const uint32_t ones[2] = {0x3C003C00u, 0x3C003C00u};  // f16 1.0 pairs
#pragma unroll
  for (int kc = 0; kc < (NBLK + 1) / 2; ++kc) {
    uint32_t pf[4];
    pf[0] = pw[2 * kc][0];
    pf[1] = pw[2 * kc][1];
    if (2 * kc + 1 < NBLK) {
      pf[2] = pw[2 * kc + 1 < NBLK ? 2 * kc + 1 : 0][0];
      pf[3] = pw[2 * kc + 1 < NBLK ? 2 * kc + 1 : 0][1];
    } else {
      pf[2] = pf[3] = 0u;
    }
    // The head's first tile starts O and the sums from zero.
#pragma unroll
    for (int nd = 0; nd < HD / 8; nd += 2) {
      uint32_t vf[4];
      ldsm_x4_t(vf, vS + kc * 16 * RB + al.v_off[nd / 2]);
      const uint32_t v0[2] = {vf[0], vf[1]}, v1[2] = {vf[2], vf[3]};
      if (FIRST && kc == 0) {
        mma_16816_f16c<true>(o[nd], pf, v0);
        mma_16816_f16c<true>(o[nd + 1], pf, v1);
      } else {
        mma_16816_f16c<false>(o[nd], pf, v0);
        mma_16816_f16c<false>(o[nd + 1], pf, v1);
      }
    }
    if (FIRST && kc == 0) mma_16816_f16c<true>(lsum, pf, ones);
    else mma_16816_f16c<false>(lsum, pf, ones);
  }
}

// One key tile of the NH heads held by a tile row block: the 8-key block
// count is resolved once, then each head's step runs in the same basic
// block (independent chains the scheduler can interleave).
template <int HD, int RB, int NH, bool FIRST, bool QF16>
__device__ __forceinline__ void attn_step_dispatch(int nkeys, uint32_t kS, uint32_t vS,
                                                   const AttnLane<HD, RB> (&al)[NH], int lane,
                                                   float scale_log2,
                                                   const uint32_t (&qf)[NH][HD / 16][4],
                                                   float (&o)[NH][HD / 8][4], float (&m)[NH][2],
                                                   float (&l)[NH][4]) {
  const int nblk = (nkeys + 7) >> 3;
  const bool partial = (nkeys & 7) != 0;
#define FUTON_STEP(NB)                                                                      \
  case NB:                                                                                  \
    if (partial) {                                                                          \
      _Pragma("unroll") for (int e = 0; e < NH; ++e)                                        \
        attn_step<HD, RB, NB, true, FIRST, QF16>(kS, vS, al[e], lane, nkeys, scale_log2,     \
                                                 qf[e], o[e], m[e], l[e]);                  \
    } else {                                                                                \
      _Pragma("unroll") for (int e = 0; e < NH; ++e)                                        \
        attn_step<HD, RB, NB, false, FIRST, QF16>(kS, vS, al[e], lane, nkeys, scale_log2,    \
                                                  qf[e], o[e], m[e], l[e]);                 \
    }                                                                                       \
    break;
  switch (nblk) {
    FUTON_STEP(1) FUTON_STEP(2) FUTON_STEP(3) FUTON_STEP(4)
    FUTON_STEP(5) FUTON_STEP(6) FUTON_STEP(7) FUTON_STEP(8)
  }
#undef FUTON_STEP
}

// grid = ntiles (or nseq in cls_mode), block = 128 (4 warps × 16 query rows).
// One CTA per 64-query tile of one sequence, looping over every head, NH
// heads per step (their q, k, v columns are adjacent in qkv, so one TMA box
// of NH·HD columns carries them); q, k, v arrive pre-rotated (RoPE runs in
// the qkv GEMM epilogue). Work stops where a sequence ends: warps whose 16
// query rows all lie past the sequence idle, and a step multiplies only the
// 8-key blocks that hold keys (most benchmark sequences are shorter than one
// 64 × 64 tile). Tile rows past the sequence hold the next sequence's
// (finite) values or TMA's zero fill past T: their keys are masked, their
// probabilities are 0 and their query rows are not stored. cls_mode: CTA s
// computes only query row 0 of sequence s (the CLS-pruned last layer) into
// row s of out. A load that does not land within the wait limit sets *err
// (kDevTimeoutAttn) and the CTA stops.
// CTAs per SM the register budget is cut for. Measured on the bge shape:
// two heads per step at 3 CTAs (168 registers) beat one head at 5 (96) by
// 2 %, and two heads at 4 (128, with spills) or one head at 6-8 were slower.
template <int HD, int NH>
constexpr int attn_heads_min_ctas() { return NH == 2 ? 3 : HD == 32 ? 5 : 4; }

// SPLIT: blockIdx.y takes an equal share of the head groups instead of all
// of them (grid.y CTAs per tile), for micro-batches whose tile count alone
// leaves most SMs idle.
template <int HD, int NH, typename OutT, bool SPLIT = false>
__global__ void __launch_bounds__(128, attn_heads_min_ctas<HD, NH>())
    attn_heads_kernel(const __grid_constant__ CUtensorMap tm_qkv, int hidden, int num_heads,
                      const int* __restrict__ cu_seqlens, const AttnTile* __restrict__ tiles,
                      int cls_mode, float scale_log2, OutT* __restrict__ out, int ldo,
                      int* __restrict__ err) {
  constexpr int W = HD * NH;  // tile width in elements
  // f16 outputs: the qkv buffer holds f16 q and k too (else bf16 q, k).
  constexpr bool kQF16 = std::is_same<OutT, __half>::value;
  using SM = AttnSmem<W>;
  constexpr int RB = SM::kRowBytes, kTile = SM::kTileBytes;
  extern __shared__ uint8_t sm_raw[];
  const uint32_t sbase = (smem_u32(sm_raw) + 1023u) & ~1023u;
  const uint32_t sQ = sbase;                              // slot = head group % ring
  const uint32_t sK = sbase + kAttnRing * kTile;          // slot = step % ring
  const uint32_t sV = sbase + 2 * kAttnRing * kTile;
  const uint32_t full = sbase + SM::kBarOffset;           // kAttnRing mbarriers
  __shared__ int abort_flag;

  const AttnTile tile = tiles[blockIdx.x];  // cls_mode: (sequence, 0)
  const int s0 = cu_seqlens[tile.seq];
  const int L = cu_seqlens[tile.seq + 1] - s0;
  const int qlim = cls_mode ? 1 : L;  // query positions < qlim are real
  const int nkv = (L + 63) / 64;
  int g_begin = 0, g_end = num_heads / NH;
  if constexpr (SPLIT) {
    const int per = (g_end + (int)gridDim.y - 1) / (int)gridDim.y;
    g_begin = (int)blockIdx.y * per;
    g_end = min(g_end, g_begin + per);
    if (g_begin >= g_end) return;  // uniform over the CTA, before any barrier
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool warp_active = tile.q0 + warp * 16 < qlim;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    tma_prefetch_desc(&tm_qkv);
#pragma unroll
    for (int i = 0; i < kAttnRing; ++i) mbar_init(full + 8 * i, 1);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();  // qkv and out only after the previous kernel has completed
  pdl_trigger();

  // Next (head group, key tile) to load (thread 0 only).
  int ng = g_begin, nj = 0, issued = 0;
  auto issue_next = [&]() {
    if (ng >= g_end) return;
    const int slot = issued % kAttnRing;
    const uint32_t bar = full + 8 * slot;
    mbar_arrive_expect_tx(bar, (nj == 0 ? 3 : 2) * kTile);
    if (nj == 0) tma_load_2d(sQ + (ng % kAttnRing) * kTile, &tm_qkv, bar, ng * W, s0 + tile.q0);
    tma_load_2d(sK + slot * kTile, &tm_qkv, bar, hidden + ng * W, s0 + nj * 64);
    tma_load_2d(sV + slot * kTile, &tm_qkv, bar, 2 * hidden + ng * W, s0 + nj * 64);
    if (++nj == nkv) { nj = 0; ++ng; }
    ++issued;
  };

  AttnLane<HD, RB> al[NH];
#pragma unroll
  for (int e = 0; e < NH; ++e) al[e] = AttnLane<HD, RB>(lane, e);
  const int qr = warp * 16 + (lane & 15);
  const uint32_t q_row = qr * RB, q_swz = attn_swz<RB>(qr), q_hi = lane >> 4;

  uint32_t qf[NH][HD / 16][4];
  float o[NH][HD / 8][4];
  float m_run[NH][2], l_run[NH][4];
  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < kAttnRing - 1; ++i) issue_next();
  }
  int step = 0;
  for (int g = g_begin; g < g_end; ++g) {
    for (int j = 0; j < nkv; ++j, ++step) {
      if (threadIdx.x == 0) issue_next();
      const int slot = step % kAttnRing;
      if (!mbar_wait_bounded(full + 8 * slot, (step / kAttnRing) & 1, err, kDevTimeoutAttn,
                             &abort_flag))
        return;
      if (warp_active) {
        const uint32_t kS = sK + slot * kTile;
        // V columns are stored as f16 by the qkv GEMM epilogue.
        const uint32_t vS = sV + slot * kTile;
        const int nkeys = min(64, L - j * 64);
        if (j == 0) {
          const uint32_t qS = sQ + (g % kAttnRing) * kTile + q_row;
#pragma unroll
          for (int e = 0; e < NH; ++e)
#pragma unroll
            for (int kc = 0; kc < HD / 16; ++kc)
              ldsm_x4(qf[e][kc], qS + (((e * (HD / 8) + 2 * kc + q_hi) ^ q_swz) << 4));
          attn_step_dispatch<HD, RB, NH, true, kQF16>(nkeys, kS, vS, al, lane, scale_log2, qf, o,
                                                      m_run, l_run);
        } else {
          attn_step_dispatch<HD, RB, NH, false, kQF16>(nkeys, kS, vS, al, lane, scale_log2, qf, o,
                                                       m_run, l_run);
        }
        if (j == nkv - 1) {
          const int qr0 = tile.q0 + warp * 16 + (lane >> 2), qr1 = qr0 + 8;
          const size_t orow0 = cls_mode ? (size_t)tile.seq : (size_t)(s0 + qr0);
          OutT* const out0 = out + orow0 * ldo + (lane & 3) * 2;
          OutT* const out1 = out + (size_t)(s0 + qr1) * ldo + (lane & 3) * 2;
#pragma unroll
          for (int e = 0; e < NH; ++e) {
            // Every column of the ones block holds the full row sum; l ≥ 1
            // (the row maximum contributes 2^0), so the approximate
            // reciprocal (≤ 1 ulp) is safe.
            const float inv0 = rcp_approx(l_run[e][0]), inv1 = rcp_approx(l_run[e][2]);
#pragma unroll
            for (int nd = 0; nd < HD / 8; ++nd) {
              const int col = (g * NH + e) * HD + nd * 8;
              if (qr0 < qlim) store2<OutT>(out0 + col, o[e][nd][0] * inv0, o[e][nd][1] * inv0);
              if (qr1 < qlim) store2<OutT>(out1 + col, o[e][nd][2] * inv1, o[e][nd][3] * inv1);
            }
          }
        }
      }
      __syncthreads();  // every warp is done with this slot before it is refilled
    }
  }
}

// Index of the sequence holding packed row `row` (cu is non-decreasing).
__device__ __forceinline__ int find_seq(const int* cu, int nseq, int row) {
  int lo = 0, hi = nseq;  // invariant: cu[lo] <= row < cu[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (cu[mid] <= row) lo = mid; else hi = mid;
  }
  return lo;
}

// One warp per (query, head). cls_mode = 0: query i is packed row i (all
// tokens); output row i. cls_mode = 1: query i is the first token of
// sequence i; output row i of a compact [nseq, ldo] buffer.
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(fminf(fmaxf(v, -65504.0f), 65504.0f));
}
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <int HD, typename InT, typename OutT>
__global__ void __launch_bounds__(256)
    attn_rowq_kernel(const InT* __restrict__ qkv, int hidden, int num_heads,
                     const int* __restrict__ cu_seqlens, int nseq, int nq, int cls_mode,
                     const float* __restrict__ rcos, const float* __restrict__ rsin, int rope,
                     float scale_log2, OutT* __restrict__ out, int ldo) {
  pdl_wait();
  pdl_trigger();
  const int gw = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  const int qi = gw / num_heads, head = gw % num_heads;
  if (qi >= nq) return;
  int seq, qrow;
  if (cls_mode) {
    seq = qi;
    qrow = cu_seqlens[qi];
  } else {
    qrow = qi;
    seq = find_seq(cu_seqlens, nseq, qi);
  }
  const int s0 = cu_seqlens[seq];
  const int L = cu_seqlens[seq + 1] - s0;
  const int qpos = qrow - s0;
  const int ld = 3 * hidden;
  constexpr int kHalf = HD / 2;

  float q[HD];
  {
    const InT* p = qkv + (size_t)qrow * ld + head * HD;
#pragma unroll
    for (int d = 0; d < HD; ++d) q[d] = to_f32(p[d]);
    if (rope) {
#pragma unroll
      for (int i = 0; i < kHalf; ++i) {
        float c = rcos[(size_t)qpos * kHalf + i], s = rsin[(size_t)qpos * kHalf + i];
        float x1 = q[i], x2 = q[i + kHalf];
        q[i] = x1 * c - x2 * s;
        q[i + kHalf] = x2 * c + x1 * s;
      }
    }
  }
  float m = -INFINITY, l = 0.f;
  float o[HD];
#pragma unroll
  for (int d = 0; d < HD; ++d) o[d] = 0.f;
  for (int j = lane; j < L; j += 32) {
    const InT* kp = qkv + (size_t)(s0 + j) * ld + hidden + head * HD;
    const InT* vp = kp + hidden;
    float k[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) k[d] = to_f32(kp[d]);
    if (rope) {
#pragma unroll
      for (int i = 0; i < kHalf; ++i) {
        float c = rcos[(size_t)j * kHalf + i], s = rsin[(size_t)j * kHalf + i];
        float x1 = k[i], x2 = k[i + kHalf];
        k[i] = x1 * c - x2 * s;
        k[i + kHalf] = x2 * c + x1 * s;
      }
    }
    float sc = 0.f;
#pragma unroll
    for (int d = 0; d < HD; ++d) sc += q[d] * k[d];
    sc *= scale_log2;
    const float m_new = fmaxf(m, sc);
    const float alpha = (m == -INFINITY) ? 0.f : exp2f(m - m_new);
    const float p = exp2f(sc - m_new);
    l = l * alpha + p;
#pragma unroll
    for (int d = 0; d < HD; ++d) o[d] = o[d] * alpha + p * to_f32(vp[d]);
    m = m_new;
  }
  const float mw = warp_max(m);
  const float a = (m == -INFINITY) ? 0.f : exp2f(m - mw);
  const float lw = warp_sum(l * a);
  const float inv = 1.f / lw;
  OutT* dst = out + (size_t)(cls_mode ? qi : qrow) * ldo + head * HD;
#pragma unroll
  for (int d = 0; d < HD; ++d) {
    const float v = warp_sum(o[d] * a);
    if (lane == (d & 31)) dst[d] = from_f32<OutT>(v * inv);
  }
}

}  // namespace futon
