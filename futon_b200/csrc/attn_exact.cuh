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
//     64-key tiles staged in shared memory, then the exponentials and their
//     f64 sum over its row of P, which lives in global scratch, key-major per
//     sequence (entry (row r, key j) of sequence s at poff[s] + j·nq + r,
//     nq = the sequence's query rows), so a warp's rows are adjacent; the
//     row's float32(1/sum) goes to a separate array;
//   attn_exact_pv_kernel  32 query rows per CTA, 2 rows × 4 output columns
//     per thread: p = e·inv formed as 64-key tiles of P are staged in shared
//     memory with V, then the chains of exact_pv_tile.
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

// The device kernels evaluate the routines above with paired f32 FMAs
// (fma.rn.f32x2: two independent fmaf, each rounded once), pairing chains
// l and l + 4 of one dot product (scores) or two adjacent output columns
// (P·V); every chain still takes its products one at a time, in the same
// order, so the results are bit-identical.

// Scores and softmaxScaled of one head group. grid = (tiles, or sequences in
// cls_mode; heads of this group), block = 64: thread i takes query row
// q0 + i of its tile's sequence; head = head0 + blockIdx.y, whose P block
// starts at P + blockIdx.y · pstride. Writes e = exp(s·scale − max·scale)
// (zeros for the padded keys) to P and inv = float32(1/Σe) to
// pinv[blockIdx.y · pinv_ld + row] (row: the query's micro-batch row, or
// its sequence in cls_mode); the P·V kernel forms p = e·inv.
// The key tile is staged with each key's 8-value groups stored as (d, d+4)
// pairs: [k0 k4 k1 k5 k2 k6 k3 k7].
template <int HD>
__global__ void __launch_bounds__(64)
    attn_exact_softmax_kernel(const float* __restrict__ qkv, int hidden, int head0,
                              const int* __restrict__ cu, const AttnTile* __restrict__ tiles,
                              int cls_mode, const int* __restrict__ poff, size_t pstride,
                              float scale, float* __restrict__ P, float* __restrict__ pinv,
                              int pinv_ld) {
  static_assert(HD % 8 == 0, "head_dim must be a multiple of 8");
  __shared__ __align__(16) float sK[kExactKeyTile * HD];
  const AttnTile tile = tiles[blockIdx.x];  // cls_mode: (sequence, 0)
  const int head = head0 + (int)blockIdx.y;
  const int s0 = cu[tile.seq], L = cu[tile.seq + 1] - s0;
  const int nq = cls_mode ? 1 : L, kp = (L + 7) & ~7;
  const int r = tile.q0 + (int)threadIdx.x;
  const bool live = r < nq;
  const size_t ld = 3 * (size_t)hidden;
  float* prow = P + (size_t)blockIdx.y * pstride + (size_t)poff[tile.seq] + (size_t)(live ? r : 0);
  // q as (d, d+4) pairs: qp[4g + i] = (q[8g + i], q[8g + i + 4]).
  uint64_t qp[HD / 2];
  if (live) {
    const float4* src = reinterpret_cast<const float4*>(qkv + (size_t)(s0 + r) * ld + head * HD);
#pragma unroll
    for (int g = 0; g < HD / 8; ++g) {
      const float4 a = src[2 * g], b = src[2 * g + 1];
      qp[4 * g] = f2_pack(a.x, b.x);
      qp[4 * g + 1] = f2_pack(a.y, b.y);
      qp[4 * g + 2] = f2_pack(a.z, b.z);
      qp[4 * g + 3] = f2_pack(a.w, b.w);
    }
  }
  float mx = 0.0f;
  for (int k0 = 0; k0 < L; k0 += kExactKeyTile) {
    const int n = min(kExactKeyTile, L - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < n * (HD / 8); i += blockDim.x) {
      const int jj = i / (HD / 8), g = i % (HD / 8);
      const float4* src =
          reinterpret_cast<const float4*>(qkv + (size_t)(s0 + k0 + jj) * ld + hidden + head * HD);
      const float4 a = src[2 * g], b = src[2 * g + 1];
      float4* dst = reinterpret_cast<float4*>(sK + (size_t)jj * HD + 8 * g);
      dst[0] = make_float4(a.x, b.x, a.y, b.y);
      dst[1] = make_float4(a.z, b.z, a.w, b.w);
    }
    __syncthreads();
    if (live) {
      for (int jj = 0; jj < n; ++jj) {
        const float4* kr = reinterpret_cast<const float4*>(sK + (size_t)jj * HD);
        uint64_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;  // chains (0,4) (1,5) (2,6) (3,7)
#pragma unroll
        for (int g = 0; g < HD / 8; ++g) {
          const float4 u = kr[2 * g], w = kr[2 * g + 1];
          a0 = f2_fma(f2_pack(u.x, u.y), qp[4 * g], a0);
          a1 = f2_fma(f2_pack(u.z, u.w), qp[4 * g + 1], a1);
          a2 = f2_fma(f2_pack(w.x, w.y), qp[4 * g + 2], a2);
          a3 = f2_fma(f2_pack(w.z, w.w), qp[4 * g + 3], a3);
        }
        float c0, c4, c1, c5, c2, c6, c3, c7;
        f2_unpack(a0, c0, c4);
        f2_unpack(a1, c1, c5);
        f2_unpack(a2, c2, c6);
        f2_unpack(a3, c3, c7);
        const float sc = fadd(fadd(fadd(c0, c4), fadd(c1, c5)), fadd(fadd(c2, c6), fadd(c3, c7)));
        prow[(size_t)(k0 + jj) * nq] = sc;
        if (k0 + jj == 0 || sc > mx) mx = sc;
      }
    }
  }
  if (!live) return;
  // softmaxScaled up to the sum (exact_softmax_row without its final
  // scaling), eight scores in flight: every load of a group is issued
  // before the group's first store (the row's scores in key order, the f64
  // sum still taken one key after another).
  const float ms = fmul(mx, scale);
  double sum = 0.0;
  constexpr int kG = 8;
  int j = 0;
  for (; j + kG <= L; j += kG) {
    float v[kG];
#pragma unroll
    for (int u = 0; u < kG; ++u) v[u] = prow[(size_t)(j + u) * nq];
#pragma unroll
    for (int u = 0; u < kG; ++u) {
      float dd = fsub(fmul(v[u], scale), ms);
      if (dd < kExpClampLo) dd = kExpClampLo;
      v[u] = exp_f32(dd);
      sum += (double)v[u];
    }
#pragma unroll
    for (int u = 0; u < kG; ++u) prow[(size_t)(j + u) * nq] = v[u];
  }
  for (; j < L; ++j) {
    float dd = fsub(fmul(prow[(size_t)j * nq], scale), ms);
    if (dd < kExpClampLo) dd = kExpClampLo;
    const float e = exp_f32(dd);
    prow[(size_t)j * nq] = e;
    sum += (double)e;
  }
  for (j = L; j < kp; ++j) prow[(size_t)j * nq] = 0.0f;
  const size_t irow = cls_mode ? (size_t)tile.seq : (size_t)(s0 + r);
  pinv[(size_t)blockIdx.y * pinv_ld + irow] = (float)(1.0 / sum);
}

// O = P·V of one head group, p = e·inv formed as P is staged. grid =
// (tiles, or sequences in cls_mode; 2 halves of 32 query rows; heads of this
// group), block = 16 · HD/4: thread t takes query rows 2·(t / (HD/4)) and
// the next of its half, and output columns 4·(t % (HD/4)) .. + 3; each of
// those 8 outputs keeps the eight chains of exact_pv_tile (key j feeds
// chain j mod 8), paired over adjacent columns.
template <int HD>
__global__ void __launch_bounds__(4 * HD)
    attn_exact_pv_kernel(const float* __restrict__ qkv, int hidden, int head0,
                         const int* __restrict__ cu, const AttnTile* __restrict__ tiles,
                         int cls_mode, const int* __restrict__ poff, size_t pstride,
                         const float* __restrict__ P, const float* __restrict__ pinv, int pinv_ld,
                         float* __restrict__ out, int ldo) {
  constexpr int kT = kExactKeyTile, kCg = HD / 4;
  __shared__ __align__(16) float sV[kT * HD];
  __shared__ __align__(16) float sP[kT * 32];  // [key][row of the half]
  __shared__ float sInv[32];
  const AttnTile tile = tiles[blockIdx.x];  // cls_mode: (sequence, 0)
  const int head = head0 + (int)blockIdx.z;
  const int s0 = cu[tile.seq], L = cu[tile.seq + 1] - s0;
  const int nq = cls_mode ? 1 : L, kp = (L + 7) & ~7;
  const int rbase = tile.q0 + 32 * (int)blockIdx.y;
  if (rbase >= nq) return;  // the whole CTA: no row of this half exists
  const int cg = (int)threadIdx.x % kCg, rp = (int)threadIdx.x / kCg;
  const int r0 = rbase + 2 * rp;
  const size_t ld = 3 * (size_t)hidden;
  const float* pblk = P + (size_t)blockIdx.z * pstride + (size_t)poff[tile.seq];
  if (threadIdx.x < 32) {
    const int rr = rbase + (int)threadIdx.x;
    const size_t irow = cls_mode ? (size_t)tile.seq : (size_t)(s0 + rr);
    sInv[threadIdx.x] = rr < nq ? pinv[(size_t)blockIdx.z * pinv_ld + irow] : 0.0f;
  }
  // acc[row][column pair][chain]: (column 4·cg + 2·c, + 1) of row r0 + row.
  uint64_t acc[2][2][8];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int l = 0; l < 8; ++l) acc[a][b][l] = 0;
  for (int k0 = 0; k0 < kp; k0 += kT) {
    const int n = min(kT, kp - k0);  // a multiple of 8
    __syncthreads();
    // V (n × HD) and P (n × 32) of the tile: every thread's loads are
    // issued before its stores (n·HD/4 and 32·n are multiples of blockDim).
    {
      constexpr int kVI = kT * (HD / 4) / (4 * HD), kPI = kT * 32 / (4 * HD);
      float4 vv[kVI];
      float pp[kPI];
#pragma unroll
      for (int u = 0; u < kVI; ++u) {
        const int i = (int)threadIdx.x + u * (int)blockDim.x;
        const int jj = i / (HD / 4), c = i % (HD / 4);
        vv[u] = (jj < n && k0 + jj < L)
                    ? reinterpret_cast<const float4*>(qkv + (size_t)(s0 + k0 + jj) * ld +
                                                      2 * hidden + head * HD)[c]
                    : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kPI; ++u) {
        const int i = (int)threadIdx.x + u * (int)blockDim.x;
        const int jj = i >> 5, qi = i & 31;
        const int rr = rbase + qi;
        pp[u] = (jj < n && rr < nq) ? pblk[(size_t)(k0 + jj) * nq + rr] : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kVI; ++u)
        reinterpret_cast<float4*>(sV)[(int)threadIdx.x + u * (int)blockDim.x] = vv[u];
#pragma unroll
      for (int u = 0; u < kPI; ++u) {
        const int i = (int)threadIdx.x + u * (int)blockDim.x;
        sP[i] = fmul(pp[u], sInv[i & 31]);
      }
    }
    __syncthreads();
    for (int j8 = 0; j8 < n; j8 += 8) {
#pragma unroll
      for (int l = 0; l < 8; ++l) {
        const int jj = j8 + l;
        const float2 p = *reinterpret_cast<const float2*>(sP + jj * 32 + 2 * rp);
        const float4 v = reinterpret_cast<const float4*>(sV + (size_t)jj * HD)[cg];
        const uint64_t v01 = f2_pack(v.x, v.y), v23 = f2_pack(v.z, v.w);
        const uint64_t p0 = f2_pack(p.x, p.x), p1 = f2_pack(p.y, p.y);
        acc[0][0][l] = f2_fma(v01, p0, acc[0][0][l]);
        acc[0][1][l] = f2_fma(v23, p0, acc[0][1][l]);
        acc[1][0][l] = f2_fma(v01, p1, acc[1][0][l]);
        acc[1][1][l] = f2_fma(v23, p1, acc[1][1][l]);
      }
    }
  }
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    const int rr = r0 + a;
    if (rr >= nq) continue;
    float y[4];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      Fma8 ca, cb;
#pragma unroll
      for (int l = 0; l < 8; ++l) f2_unpack(acc[a][b][l], ca.c[l], cb.c[l]);
      y[2 * b] = ca.fold();
      y[2 * b + 1] = cb.fold();
    }
    const size_t orow = cls_mode ? (size_t)tile.seq : (size_t)(s0 + rr);
    *reinterpret_cast<float4*>(out + orow * (size_t)ldo + head * HD + 4 * cg) =
        make_float4(y[0], y[1], y[2], y[3]);
  }
}

#endif  // FUTON_EXACT_KERNELS

}  // namespace futon
