// attn_exact.cuh — the int8 path's attention in the reference's exact
// float32 operation order: attendHead and softmaxScaled
// (native/model.go:646-739) with the avx2Kernel MatMulT that runs the
// attention products of the reference's default amd64 build
// (native/kernel_avx2_amd64.go:47-90, kernel_avx2_amd64.s:20-111).
//
// The int8 forward quantises every layer's activations per row
// (native/quant.go:42-70), and a row's codes move by a whole step wherever a
// value crosses a rounding boundary, so float32-rounding-level differences in
// the attention output grow into visible vector differences. This path
// therefore repeats the reference's float32 operations one for one:
//   S = q·kᵀ and O = P·V: every output element is eight fused multiply-add
//     chains (chain l takes the products of indices p ≡ l mod 8, in
//     increasing p) folded as ((c0 + c4) + (c1 + c5)) + ((c2 + c6) + (c3 + c7)),
//     the eight-lane FMA accumulators of the dot4x2f32 panel and its REDUCE1
//     fold; the keys are padded to a multiple of 8 with zeros (padSeq,
//     model.go:532), and the padded products take part in the chains;
//   softmaxScaled: the maximum of the sequence's raw scores times the scale,
//     d = s·scale − max·scale with two roundings, a clamp at −104, Cephes
//     expF32 (exp_f32), a float64 running sum in key order, inv =
//     float32(1/sum) and p = e·inv.
// Queries and keys arrive rotated by the qkv GEMM epilogue, which rounds
// rotateHalf's products and sums separately on this path.
//
// Kernels (float32 qkv [T, 3h] in, float32 [rows, h] out), per head group:
//   attn_exact_softmax_kernel  one thread per query row: its scores against
//     64-key tiles staged in shared memory, then the softmax over its row of
//     P, which lives in global scratch, key-major per sequence (entry
//     (row r, key j) of sequence s at poff[s] + j·nq + r, nq = the sequence's
//     query rows), so a warp's rows are adjacent;
//   attn_exact_pv_kernel  16 query rows × 16 column groups per CTA: each
//     thread folds HD/16 output columns of one row over 64-key tiles of P
//     and V staged in shared memory.
// Both serve the CLS-pruned last layer (model.go:403-410) too: one query row
// per sequence, written to row s of a compact output.
#pragma once

#include <cmath>

#include "mathf32.cuh"
// FUTON_EXACT_HOST_ONLY: the arithmetic routines without the kernels (a host
// test build of them).
#if defined(__CUDACC__) && !defined(FUTON_EXACT_HOST_ONLY)
#define FUTON_EXACT_KERNELS 1
#include "attention.cuh"
#endif

namespace futon {

// Eight FMA accumulation chains and the fold of the dot4x2f32 panel.
struct Fma8 {
  float c[8];
  FUTON_HD __forceinline__ void zero() {
#pragma unroll
    for (int l = 0; l < 8; ++l) c[l] = 0.0f;
  }
  FUTON_HD __forceinline__ float fold() const {
    return fadd(fadd(fadd(c[0], c[4]), fadd(c[1], c[5])), fadd(fadd(c[2], c[6]), fadd(c[3], c[7])));
  }
};

// q·k over HD values (HD a multiple of 8: no scalar tail).
template <int HD>
FUTON_HD __forceinline__ float exact_dot(const float* q, const float* k) {
  static_assert(HD % 8 == 0, "head_dim must be a multiple of 8");
  Fma8 a;
  a.zero();
#pragma unroll
  for (int d = 0; d < HD; ++d) a.c[d & 7] = fmaf(k[d], q[d], a.c[d & 7]);
  return a.fold();
}

// Scores of one query row against n staged keys (key j0 + j at kt + j·HD):
// written to prow[(j0 + j)·stride], running maximum in *mx (first key sets it).
template <int HD>
FUTON_HD __forceinline__ void exact_scores_tile(const float* q, const float* kt, int n, int j0,
                                                float* prow, size_t stride, float* mx) {
  for (int j = 0; j < n; ++j) {
    const float s = exact_dot<HD>(q, kt + (size_t)j * HD);
    prow[(size_t)(j0 + j) * stride] = s;
    if (j0 + j == 0 || s > *mx) *mx = s;
  }
}

// softmaxScaled over the L raw scores of one row (prow[j·stride]), then the
// padded keys [L, kp) set to zero.
FUTON_HD __forceinline__ void exact_softmax_row(float* prow, size_t stride, int L, int kp,
                                                float scale, float mx) {
  const float ms = fmul(mx, scale);
  double sum = 0.0;
  for (int j = 0; j < L; ++j) {
    float d = fsub(fmul(prow[(size_t)j * stride], scale), ms);
    if (d < kExpClampLo) d = kExpClampLo;
    const float e = exp_f32(d);
    prow[(size_t)j * stride] = e;
    sum += (double)e;
  }
  const float inv = (float)(1.0 / sum);
  for (int j = 0; j < L; ++j) prow[(size_t)j * stride] = fmul(prow[(size_t)j * stride], inv);
  for (int j = L; j < kp; ++j) prow[(size_t)j * stride] = 0.0f;
}

// Folds n keys (a multiple of 8, starting at a multiple of 8) of P·V into
// the chains of KD output columns: p[j] is this row's probability of key j,
// v + j·HD the key's value row, columns col0 + 16·i.
template <int HD, int KD>
FUTON_HD __forceinline__ void exact_pv_tile(Fma8 (&acc)[KD], const float* p, const float* v, int n,
                                            int col0) {
  for (int j8 = 0; j8 < n; j8 += 8) {
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      const float pv = p[j8 + l];
      const float* vr = v + (size_t)(j8 + l) * HD + col0;
#pragma unroll
      for (int i = 0; i < KD; ++i) acc[i].c[l] = fmaf(vr[16 * i], pv, acc[i].c[l]);
    }
  }
}

#if defined(FUTON_EXACT_KERNELS)

constexpr int kExactKeyTile = 64;

// grid = (tiles, or sequences in cls_mode; heads of this group), block = 64.
// Thread i takes query row q0 + i of its tile's sequence; head = head0 +
// blockIdx.y, whose P block starts at P + blockIdx.y · pstride.
template <int HD>
__global__ void __launch_bounds__(64)
    attn_exact_softmax_kernel(const float* __restrict__ qkv, int hidden, int head0,
                              const int* __restrict__ cu, const AttnTile* __restrict__ tiles,
                              int cls_mode, const int* __restrict__ poff, size_t pstride,
                              float scale, float* __restrict__ P) {
  __shared__ __align__(16) float sK[kExactKeyTile * HD];
  const AttnTile tile = cls_mode ? AttnTile{(int)blockIdx.x, 0} : tiles[blockIdx.x];
  const int head = head0 + (int)blockIdx.y;
  const int s0 = cu[tile.seq], L = cu[tile.seq + 1] - s0;
  const int nq = cls_mode ? 1 : L, kp = (L + 7) & ~7;
  const int r = tile.q0 + (int)threadIdx.x;
  const bool live = r < nq;
  const size_t ld = 3 * (size_t)hidden;
  float* prow = P + (size_t)blockIdx.y * pstride + (size_t)poff[tile.seq] + (size_t)(live ? r : 0);
  float q[HD];
  if (live) {
    const float4* src = reinterpret_cast<const float4*>(qkv + (size_t)(s0 + r) * ld + head * HD);
#pragma unroll
    for (int c = 0; c < HD / 4; ++c) {
      const float4 v = src[c];
      q[4 * c] = v.x;
      q[4 * c + 1] = v.y;
      q[4 * c + 2] = v.z;
      q[4 * c + 3] = v.w;
    }
  }
  float mx = 0.0f;
  for (int k0 = 0; k0 < L; k0 += kExactKeyTile) {
    const int n = min(kExactKeyTile, L - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < n * (HD / 4); i += blockDim.x) {
      const int j = i / (HD / 4), c = i % (HD / 4);
      reinterpret_cast<float4*>(sK)[i] = reinterpret_cast<const float4*>(
          qkv + (size_t)(s0 + k0 + j) * ld + hidden + head * HD)[c];
    }
    __syncthreads();
    if (live) exact_scores_tile<HD>(q, sK, n, k0, prow, (size_t)nq, &mx);
  }
  if (live) exact_softmax_row(prow, (size_t)nq, L, kp, scale, mx);
}

// grid = (tiles, or sequences in cls_mode; 4 row groups of 16; heads of this
// group), block = 256: thread t takes query row q0 + 16·blockIdx.y + t/16
// and output columns (t % 16) + 16·i of head head0 + blockIdx.z.
template <int HD>
__global__ void __launch_bounds__(256)
    attn_exact_pv_kernel(const float* __restrict__ qkv, int hidden, int head0,
                         const int* __restrict__ cu, const AttnTile* __restrict__ tiles,
                         int cls_mode, const int* __restrict__ poff, size_t pstride,
                         const float* __restrict__ P, float* __restrict__ out, int ldo) {
  constexpr int kD = HD / 16, kT = kExactKeyTile, kPs = kT + 1;
  __shared__ __align__(16) float sV[kT * HD];
  __shared__ float sP[16 * kPs];
  const AttnTile tile = cls_mode ? AttnTile{(int)blockIdx.x, 0} : tiles[blockIdx.x];
  const int head = head0 + (int)blockIdx.z;
  const int s0 = cu[tile.seq], L = cu[tile.seq + 1] - s0;
  const int nq = cls_mode ? 1 : L, kp = (L + 7) & ~7;
  const int rbase = tile.q0 + 16 * (int)blockIdx.y;
  if (rbase >= nq) return;  // the whole CTA: no row of this group exists
  const int qq = (int)threadIdx.x >> 4, g = (int)threadIdx.x & 15;
  const int r = rbase + qq;
  const bool live = r < nq;
  const size_t ld = 3 * (size_t)hidden;
  const float* pblk = P + (size_t)blockIdx.z * pstride + (size_t)poff[tile.seq];
  Fma8 acc[kD];
#pragma unroll
  for (int i = 0; i < kD; ++i) acc[i].zero();
  for (int k0 = 0; k0 < kp; k0 += kT) {
    const int n = min(kT, kp - k0);  // a multiple of 8
    __syncthreads();
    for (int i = threadIdx.x; i < n * (HD / 4); i += blockDim.x) {
      const int j = i / (HD / 4), c = i % (HD / 4);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + j < L)
        v = reinterpret_cast<const float4*>(qkv + (size_t)(s0 + k0 + j) * ld + 2 * hidden +
                                            head * HD)[c];
      reinterpret_cast<float4*>(sV)[i] = v;
    }
    for (int i = threadIdx.x; i < 16 * n; i += blockDim.x) {
      const int j = i >> 4, qi = i & 15;
      const int rr = rbase + qi;
      sP[qi * kPs + j] = rr < nq ? pblk[(size_t)(k0 + j) * nq + rr] : 0.0f;
    }
    __syncthreads();
    if (live) exact_pv_tile<HD, kD>(acc, sP + qq * kPs, sV, n, g);
  }
  if (live) {
    const size_t orow = cls_mode ? (size_t)tile.seq : (size_t)(s0 + r);
    float* dst = out + orow * (size_t)ldo + head * HD + g;
#pragma unroll
    for (int i = 0; i < kD; ++i) dst[16 * i] = acc[i].fold();
  }
}

#endif  // FUTON_EXACT_KERNELS

}  // namespace futon
