// gemm_tc.cuh — tcgen05 tensor-core GEMM for sm_100a with fused epilogues.
//
// Computes the Kernel.MatMulT contract of futon (native/kernel.go:26-36):
//     D[m, n] = Σ_k A[m, k] · W[n, k]  (+ bias[n])
// with A row-major [M, K] (activations) and W row-major [N, K] (nn.Linear
// layout, exactly how pack weights are stored), then applies one of the
// layer epilogues of native/model.go:550-635 before the single store:
//   kEpiStore   D + bias                               (qkv projection)
//   kEpiRope    D + bias, NeoX RoPE on the q/k columns (qkv of a RoPE pack)
//   kEpiGelu    gelu(D + bias)                         (fc1, model.go:610-616)
//   kEpiSwiglu  (D_fc1 + b1) * silu(D_gate + b2)       (fc1‖gate, model.go:617-627)
//   kEpiResid   (D + bias) + residual                  (out / fc2 before LayerNorm)
//   kEpiResidLN LayerNorm((D + bias) + residual)       (out / fc2 + norm1 / norm2,
//               192-column row slices in clusters, model.go:596-599, 628-633)
// and, for the int8 path (native/quant.go:99-137), the exact rescale
//   float32(sum_s32) * (scale_a[m] * scale_w[n]) + bias[n].
//
// Structure: one persistent CTA per SM, 2 + EW warps (EW = 8, or 16 for the
// bf16 GELU / plain-store tiles of width 256).
//   warp 0     TMA producer: 128-byte-swizzled K-major tiles of A (128 rows)
//              and W (BN rows) into a shared-memory ring whose depth is what
//              the shared-memory budget leaves after the epilogue's buffers.
//   warp 1     allocates tensor memory; lane 0 issues tcgen05.mma
//              (M=128, N≤256, K=16 bf16 / 32 s8 per instruction) into one of
//              two TMEM accumulators and commits completion to mbarriers.
//   warps 2-   epilogue: tcgen05.ld of the accumulator lane quarter the warp
//              may access (one output row per thread; the EW/4 warps of a
//              quarter split the 32-column chunks), fused math (paired f32
//              lanes), then either a TMA tile store through a per-warp
//              64B-swizzled staging ring (bf16 outputs: full-sector writes,
//              no per-thread stores) or direct vector stores (f32 outputs).
// The two accumulators let the epilogue of tile i overlap the MMAs of tile
// i+1. Tiles are visited n-fastest so CTAs running together share A tiles
// through L2; the weights (≤ 19 MB) stay L2-resident. The fused LayerNorm
// GEMMs run as clusters of hidden/192 CTAs, one 192-column slice each, which
// exchange per-row statistics through distributed shared memory.
// PAIR (opt-in): 256-row tiles over a CTA pair, tcgen05.mma.cta_group::2
// issued by the pair's even CTA; each CTA stages its own 128 rows of A and
// half of the tile's W rows (no multicast), commits arrive in both CTAs.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "mathf32.cuh"

namespace futon {

enum EpiKind : int {
  kEpiStore = 0, kEpiGelu = 1, kEpiSwiglu = 2, kEpiResid = 3, kEpiResidLN = 4, kEpiRope = 5,
  // kEpiResidLN reading the residual from global memory (prefetched two
  // chunks ahead) instead of a TMA-loaded shared tile: the freed 48 KB buy a
  // fourth pipeline stage for long-K GEMMs (chosen by the launcher).
  kEpiResidLNG = 6
};

struct EpiParams {
  void* out;             // bf16 or f32 output, row stride ldo elements
  int ldo;
  const float* bias;     // [N] (interleaved like W for kEpiSwiglu) or null
  const void* resid;     // kEpiResid / kEpiResidLN: [M, ldr], f32, bf16 or f16 (resid_kind)
  int ldr;
  int resid_kind;        // kResidF32, kResidBf16 or kResidF16
  const float* a_scale;  // int8 path: per-row activation scales [M]
  const float* w_scale;  // int8 path: per-row weight scales [N]
  const float* ln_w;     // kEpiResidLN: LayerNorm γ, β [N], eps
  const float* ln_b;
  float eps;
  float* out_f32;        // kEpiResidLN: optional f32 copy of the normalised rows
  // kEpiRope (the qkv projection of a RoPE pack): NeoX rotation of the q
  // and k columns (< rope_cols) per head of rope_hd, at each row's position
  // in its sequence (cu_seqlens[nseq+1]), before the store (model.go:674-685).
  const float* rope_cos;  // [positions, rope_hd/2]
  const float* rope_sin;
  int rope_hd;
  int rope_cols;
  const int* cu;
  int nseq;
  int f16_from;  // TMA-store outputs at columns ≥ f16_from are written as f16 (qkv: V)
};

enum ResidKind : int { kResidF32 = 0, kResidBf16 = 1, kResidF16 = 2 };

// Peer slots per tile parity in the LayerNorm row-statistics exchange: at
// most 4 CTAs (N ≤ 4 · 192 columns) share a row tile.
constexpr int kLnPeerSlots = 4;

// LNS: the fused residual + LayerNorm configuration (BN = 192 column slices
// in clusters): three stages, the row-statistics exchange buffer and the
// residual tile (TMA-loaded, 128 rows × BN bf16 as BN/64 swizzled 16 KB
// sub-tiles) in shared memory.
// EW: epilogue warps (a multiple of 4; EW / 4 of them share each TMEM lane
// quarter, splitting its 32-column chunks). The stage count is what the
// shared-memory budget leaves after the epilogue's buffers.
// PAIR: the tile's MMAs span a CTA pair (cta_group::2, M = 256): each CTA
// stages its own 128 rows of A and half (BN / 2 rows) of the tile's W.
template <int BN, bool S8, bool LNS = false, int EW = 8, bool RSM = true, bool PAIR = false>
struct GemmCfg {
  static constexpr int kBM = 128;                             // rows per CTA
  static constexpr int kTileM = PAIR ? 256 : 128;             // rows per tile
  static constexpr int kRowBytes = 128;                       // one swizzle row
  static constexpr int kBK = S8 ? 128 : 64;                   // elements per k-block
  static constexpr int kABytes = kBM * kRowBytes;
  static constexpr int kBRows = PAIR ? BN / 2 : BN;           // W rows staged per CTA
  static constexpr int kBBytes = kBRows * kRowBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kMmaN = BN;                            // N of one tcgen05.mma (≤ 256)
  static constexpr int kNumAcc = 2;                           // TMEM accumulators
  static constexpr uint32_t kAccStride = (BN <= 64) ? 64 : (BN <= 128) ? 128 : 256;
  static constexpr uint32_t kTmemCols = kNumAcc * kAccStride; // power of two, ≤ 512
  static constexpr int kEpiWarps = EW;
  static constexpr int kParts = EW / 4;                       // epilogue warps per lane quarter
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  // After the stage ring: barriers (≤ 1 KB), then either the LayerNorm
  // partial sums (2 × 128 double2) and one 2 KB staging buffer per epilogue
  // warp, or the TMA-store staging (per epilogue warp two 32 × 64-byte
  // buffers).
  // LayerNorm: [2 tile parities][kParts][128 rows] double2 partial sums,
  // then one 2 KB staging buffer per epilogue warp.
  static constexpr int kRedBytes = LNS ? 2 * kParts * 128 * 16 : 0;
  static constexpr int kStagingBytes = LNS ? kRedBytes + kEpiWarps * 2048 : kEpiWarps * 2 * 2048;
  static constexpr int kXchBytes = LNS ? 2 * kLnPeerSlots * 128 * 16 : 0;
  static constexpr int kResidBytes = (LNS && RSM) ? kBM * BN * 2 : 0;
  static constexpr int kColsBytes = LNS ? 3 * BN * 4 : 0;
  static constexpr int kFixedBytes =
      1024 /*barriers*/ + kStagingBytes + kXchBytes + kResidBytes + kColsBytes + 1024 /*align*/;
  static constexpr int kBudget = 227 * 1024;
  static constexpr int kFit = (kBudget - kFixedBytes) / kStageBytes;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  static constexpr int kExtraOffset = kStages * kStageBytes + 1024;  // 1024-aligned
  static constexpr int kXchOffset = kExtraOffset + kStagingBytes;
  static constexpr int kResidOffset = kXchOffset + kXchBytes;       // 1024-aligned
  // LNS: the slice's bias, γ and β (3 × BN f32), read by every tile.
  static constexpr int kColsOffset = kResidOffset + kResidBytes;
  static constexpr int kSmemBytes = kColsOffset + kColsBytes + 1024 /*align*/;
  static_assert(BN <= 256, "one tcgen05.mma covers the tile's N");
  static_assert(!PAIR || (!S8 && (BN / 2) % 16 == 0), "pair tiles: 16-bit operands, N / 2 in 16s");
  static_assert(!LNS || BN % 64 == 0, "residual sub-tiles are 64 columns wide");
  static_assert(!LNS || (BN / 32) % kParts == 0, "LayerNorm column shares are whole chunks");
  static_assert(kStages >= 3 && kSmemBytes <= kBudget, "shared-memory budget");
};

// Epilogue warps of an instantiation: 16 (two 32-column chunks each) for the
// bf16 GELU and plain-store tiles at BN 256, whose epilogues set the pace,
// and 8 otherwise (12 measured slower for the LayerNorm slices and no faster
// for the BN 192 qkv tiles).
template <int BN, int EPI, bool S8>
__host__ __device__ constexpr int gemm_epi_warps() {
  return ((EPI == kEpiGelu || EPI == kEpiStore) && !S8 && BN == 256) ? 16 : 8;
}

template <typename T> __device__ __forceinline__ void store32(T* dst, const float (&v)[32]);

template <> __device__ __forceinline__ void store32<float>(float* dst, const float (&v)[32]) {
  float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int i = 0; i < 8; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// f16 with saturation: values beyond ±65504 clamp instead of becoming inf,
// so a probability of 0 times any stored value stays 0.
__device__ __forceinline__ uint4 pack8_f16(const float* v) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(w[j]) : "f"(v[2 * j + 1]), "f"(v[2 * j]));
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ uint4 pack8_bf16(const float* v) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
    w[j] = *reinterpret_cast<uint32_t*>(&p);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <> __device__ __forceinline__ void store32<__nv_bfloat16>(__nv_bfloat16* dst,
                                                                   const float (&v)[32]) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d4[i] = pack8_bf16(v + 8 * i);
}

template <> __device__ __forceinline__ void store32<__half>(__half* dst, const float (&v)[32]) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d4[i] = pack8_f16(v + 8 * i);
}

template <typename T> __device__ __forceinline__ void store1(T* dst, float v);
template <> __device__ __forceinline__ void store1<float>(float* dst, float v) { *dst = v; }
template <> __device__ __forceinline__ void store1<__nv_bfloat16>(__nv_bfloat16* dst, float v) {
  *dst = __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ void store1<__half>(__half* dst, float v) {
  *dst = __float2half_rn(fminf(fmaxf(v, -65504.0f), 65504.0f));
}

// Two 16-bit values of one 32-bit word (low half first) as f32: f16 (F16)
// or bf16.
template <bool F16>
__device__ __forceinline__ void unpack2_16(uint32_t w, float& lo, float& hi) {
  if constexpr (F16) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
    lo = f.x;
    hi = f.y;
  } else {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xFFFF0000u);
  }
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- TMA tile store (shared → global), bulk-group completion ----------------
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Destination of one epilogue warp's 32 × 32 output chunks.
// TmaSink (bf16 outputs): each lane writes its row's 64 bytes into a
// 64B-swizzled staging buffer (16-byte chunk c of row r at c ^ ((r >> 1) & 3),
// CU_TENSOR_MAP_SWIZZLE_64B), then lane 0 stores the 32-row box with TMA;
// two buffers per warp alternate so the next chunk overlaps the store. The
// tensor map clips rows ≥ M and columns ≥ N.
template <int NBUF>
struct TmaSink {
  uint8_t* buf;              // NBUF × 2048 bytes, 1024-aligned
  const CUtensorMap* map;
  int lane;
  int count;
  int f16_from;              // columns ≥ f16_from are packed as f16
  __device__ __forceinline__ void put(const float (&v)[32], int col, int row0) {
    uint8_t* b = buf + (count % NBUF) * 2048;
    if (lane == 0 && count >= NBUF) {
      if constexpr (NBUF == 2) bulk_wait_read1(); else bulk_wait_read0();
    }
    __syncwarp();
    const int sw = (lane >> 1) & 3;
    if (col >= f16_from) {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(b + lane * 64 + ((c ^ sw) << 4)) = pack8_f16(v + 8 * c);
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(b + lane * 64 + ((c ^ sw) << 4)) = pack8_bf16(v + 8 * c);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map, smem_u32(b), col, row0);
      bulk_commit();
    }
    ++count;
  }
  __device__ __forceinline__ void drain() {
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
};

// DirectSink (f32 outputs): per-thread vector stores with bounds checks.
template <typename OutT>
struct DirectSink {
  OutT* out;
  int ldo;
  int row;
  bool row_ok;
  int ncols;
  __device__ __forceinline__ void put(const float (&v)[32], int col, int /*row0*/) {
    if (!row_ok) return;
    OutT* dst = out + (size_t)row * ldo + col;
    if (col + 32 <= ncols) {
      store32<OutT>(dst, v);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col + i < ncols) store1<OutT>(dst + i, v[i]);
    }
  }
  __device__ __forceinline__ void drain() {}
};

// 32 consecutive residual values of one row (f32 or bf16).
__device__ __forceinline__ void load_resid32(const EpiParams& ep, int row, int col, float (&r)[32]) {
  if (ep.resid_kind != kResidF32) {
    const uint4* rp = reinterpret_cast<const uint4*>(
        reinterpret_cast<const uint16_t*>(ep.resid) + (size_t)row * ep.ldr + col);
    const bool f16 = ep.resid_kind == kResidF16;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 q = rp[i];
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (f16) unpack2_16<true>(w[j], r[8 * i + 2 * j], r[8 * i + 2 * j + 1]);
        else unpack2_16<false>(w[j], r[8 * i + 2 * j], r[8 * i + 2 * j + 1]);
      }
    }
  } else {
    const float4* rp =
        reinterpret_cast<const float4*>(reinterpret_cast<const float*>(ep.resid) + (size_t)row * ep.ldr + col);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 q = rp[i];
      r[4 * i] = q.x; r[4 * i + 1] = q.y; r[4 * i + 2] = q.z; r[4 * i + 3] = q.w;
    }
  }
}

// 32 consecutive entries of a per-column f32 vector (bias, scales), zero past
// `limit` (16-byte vector loads on full chunks).
__device__ __forceinline__ void load_col32(const float* p, int col, int limit, float (&r)[32]) {
  if (!p) {
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = 0.0f;
    return;
  }
  if (col + 32 <= limit) {
    const float4* p4 = reinterpret_cast<const float4*>(p + col);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 q = p4[i];
      r[4 * i] = q.x; r[4 * i + 1] = q.y; r[4 * i + 2] = q.z; r[4 * i + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = col + i < limit ? p[col + i] : 0.0f;
  }
}

// Accumulator chunk → f32 values before the activation: f32 sum + bias, or
// the int8 rescale float32(sum) * (sA * sW) + bias (quant.go:132-135). The
// column vectors are fetched (acc_fetch) before the epilogue waits for its
// TMEM load, so the two latencies overlap, then applied (acc_apply).
template <bool S8>
struct AccCols {
  float b[32];
  float ws[S8 ? 32 : 1];
};

template <bool S8>
__device__ __forceinline__ void acc_fetch(const EpiParams& ep, int col, int N, AccCols<S8>& k) {
  load_col32(ep.bias, col, N, k.b);
  if constexpr (S8) load_col32(ep.w_scale, col, N, k.ws);
}

template <bool S8>
__device__ __forceinline__ void acc_apply(const uint32_t (&u)[32], float a_s, const EpiParams& ep,
                                          const AccCols<S8>& k, float (&v)[32]) {
  if constexpr (S8) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = fmul((float)(int32_t)u[i], fmul(a_s, k.ws[i]));
    if (ep.bias) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fadd(v[i], k.b[i]);
    }
  } else if (ep.bias) {
    // f32 sum + bias, two columns per instruction.
#pragma unroll
    for (int i = 0; i < 16; ++i)
      f2_unpack(f2_add(f2_pack(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1])),
                       f2_pack(k.b[2 * i], k.b[2 * i + 1])),
                v[2 * i], v[2 * i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(u[i]);
  }
}

// Activations: the reference's exact f32 evaluation on the int8 path (whose
// outputs are re-quantised, so every bit matters), fast forms on the bf16 path.
template <bool S8> __device__ __forceinline__ float act_gelu(float x) {
  if constexpr (S8) return gelu_f32(x); else return gelu_fast(x);
}
template <bool S8> __device__ __forceinline__ float act_silu(float g) {
  if constexpr (S8) return fmul(g, sigmoid_f32(g)); else return silu_fast(g);
}

// Position of packed row `row` within its sequence (cu non-decreasing).
__device__ __forceinline__ int seq_position(const int* cu, int nseq, int row) {
  int lo = 0, hi = nseq;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (cu[mid] <= row) lo = mid; else hi = mid;
  }
  return row - cu[lo];
}

// One NeoX rotation pair of the int8 path (rotateHalf, model.go:703-712):
// each product and sum rounded separately, as the reference does.
__device__ __forceinline__ void rope_pair_exact(float& x1, float& x2, float c, float sn) {
  const float a = x1, b = x2;
  x1 = fsub(fmul(a, c), fmul(b, sn));
  x2 = fadd(fmul(b, c), fmul(a, sn));
}

// Rotates the 32 values of one chunk in place: heads of HD ≤ 32 lie inside
// the chunk (pairs i, i + HD/2 of each head). EXACT: rope_pair_exact.
template <int HD, bool EXACT>
__device__ __forceinline__ void rope_in_chunk(float (&v)[32], const float* cr, const float* sr) {
  constexpr int kHalf = HD / 2;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if ((i % HD) < kHalf) {
      if constexpr (EXACT) {
        rope_pair_exact(v[i], v[i + kHalf], cr[i % HD], sr[i % HD]);
      } else {
        const float c = cr[i % HD], sn = sr[i % HD];
        const float x1 = v[i], x2 = v[i + kHalf];
        v[i] = x1 * c - x2 * sn;
        v[i + kHalf] = x2 * c + x1 * sn;
      }
    }
  }
}

// kEpiStore / kEpiRope / kEpiGelu / kEpiSwiglu / kEpiResid for one thread (= one row).
// The two warps sharing a TMEM lane quarter split the 32-column chunks
// (part = 0/1; whole heads per thread when RoPE is on).
template <int BN, int EPI, bool S8, int kParts, typename Sink>
__device__ __forceinline__ void epilogue_row(uint32_t taddr, int row, int row0, int M, int N,
                                             int nb, int part, const EpiParams& ep, Sink& sink) {
  const bool row_ok = row < M;
  const float a_s = (S8 && row_ok) ? ep.a_scale[row] : 0.0f;
  if constexpr (EPI == kEpiSwiglu) {
    constexpr int kHalf = BN / 2;
    const int wcol0 = nb * BN;            // interleaved weight/bias column of this tile
    const int ocol0 = nb * kHalf;         // output column of this tile
#pragma unroll 1
    for (int c = 32 * part; c < kHalf; c += 32 * kParts) {
      uint32_t u[32], g[32];
      tmem_ld32(taddr + c, u);
      tmem_ld32(taddr + kHalf + c, g);
      float hv[32], gv[32], v[32];
      {
        AccCols<S8> k;
        acc_fetch<S8>(ep, wcol0 + c, N, k);
        tmem_ld_wait();
        acc_apply<S8>(u, a_s, ep, k, hv);
      }
      {
        AccCols<S8> k;
        acc_fetch<S8>(ep, wcol0 + kHalf + c, N, k);
        acc_apply<S8>(g, a_s, ep, k, gv);
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fmul(hv[i], act_silu<S8>(gv[i]));
      sink.put(v, ocol0 + c, row0);
    }
  } else if constexpr (EPI == kEpiStore || EPI == kEpiRope) {
    const int col0 = nb * BN;
    constexpr bool rope = EPI == kEpiRope;
    const int hd = ep.rope_hd, half = hd >> 1;
    const int pos = (rope && row_ok) ? seq_position(ep.cu, ep.nseq, row) : 0;
    const float* cr = rope ? ep.rope_cos + (size_t)pos * half : nullptr;
    const float* sr = rope ? ep.rope_sin + (size_t)pos * half : nullptr;
    if (rope && hd == 64) {
      // A head's two halves are two 32-column chunks: heads alternate by part.
#pragma unroll 1
      for (int c = 64 * part; c < BN; c += 64 * kParts) {
        float a[32], b[32];
        {
          uint32_t u[32];
          tmem_ld32(taddr + c, u);
          AccCols<S8> k;
          acc_fetch<S8>(ep, col0 + c, N, k);
          tmem_ld_wait();
          acc_apply<S8>(u, a_s, ep, k, a);
        }
        {
          uint32_t u[32];
          tmem_ld32(taddr + c + 32, u);
          AccCols<S8> k;
          acc_fetch<S8>(ep, col0 + c + 32, N, k);
          tmem_ld_wait();
          acc_apply<S8>(u, a_s, ep, k, b);
        }
        if (col0 + c < ep.rope_cols) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if constexpr (S8) {
              rope_pair_exact(a[i], b[i], cr[i], sr[i]);
            } else {
              const float x1 = a[i], x2 = b[i], cc = cr[i], sn = sr[i];
              a[i] = x1 * cc - x2 * sn;
              b[i] = x2 * cc + x1 * sn;
            }
          }
        }
        sink.put(a, col0 + c, row0);
        sink.put(b, col0 + c + 32, row0);
      }
    } else if constexpr (!rope && !S8 && BN % (32 * kParts) == 0) {
      // The next chunk's TMEM load is in flight while this one is processed.
      constexpr int kPer = BN / (32 * kParts);
      uint32_t ub[2][32];
      tmem_ld32(taddr + 32 * part, ub[0]);
#pragma unroll
      for (int q = 0; q < kPer; ++q) {
        const int c = 32 * (part + q * kParts);
        AccCols<S8> k;
        acc_fetch<S8>(ep, col0 + c, N, k);
        tmem_ld_wait();
        if (q + 1 < kPer) tmem_ld32(taddr + c + 32 * kParts, ub[(q + 1) & 1]);
        float v[32];
        acc_apply<S8>(ub[q & 1], a_s, ep, k, v);
        sink.put(v, col0 + c, row0);
      }
    } else {
#pragma unroll 1
      for (int c = 32 * part; c < BN; c += 32 * kParts) {
        uint32_t u[32];
        tmem_ld32(taddr + c, u);
        AccCols<S8> k;
        acc_fetch<S8>(ep, col0 + c, N, k);
        tmem_ld_wait();
        float v[32];
        acc_apply<S8>(u, a_s, ep, k, v);
        if (rope && col0 + c < ep.rope_cols) {
          if (hd == 32) rope_in_chunk<32, S8>(v, cr, sr);
          else if (hd == 16) rope_in_chunk<16, S8>(v, cr, sr);
          else rope_in_chunk<8, S8>(v, cr, sr);
        }
        sink.put(v, col0 + c, row0);
      }
    }
  } else {
    const int col0 = nb * BN;
#pragma unroll 1
    for (int c = 32 * part; c < BN; c += 32 * kParts) {
      uint32_t u[32];
      tmem_ld32(taddr + c, u);
      const int col = col0 + c;
      float r[32];
      if constexpr (EPI == kEpiResid) {
        if (row_ok && col + 32 <= N) {
          load_resid32(ep, row, col, r);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0.0f;
        }
      }
      AccCols<S8> k;
      acc_fetch<S8>(ep, col, N, k);
      tmem_ld_wait();
      float v[32];
      acc_apply<S8>(u, a_s, ep, k, v);
      if constexpr (EPI == kEpiGelu && !S8) {
#pragma unroll
        for (int i = 0; i < 16; ++i) gelu_fast2(v[2 * i], v[2 * i + 1]);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if constexpr (EPI == kEpiGelu) v[i] = act_gelu<S8>(v[i]);
          if constexpr (EPI == kEpiResid) v[i] = fadd(v[i], r[i]);
        }
      }
      sink.put(v, col, row0);
    }
  }
}

__device__ __forceinline__ float4 ld_shared_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}

// Row-statistics exchange between the CTAs of a cluster that hold the column
// slices of one row tile (peers = N / BN; 1 = no exchange).
struct LnPeers {
  int peers;
  uint32_t rank;     // this CTA's slice; slice r of the same rows is cluster rank r·rstride + rhalf
  uint32_t rstride, rhalf;
  uint32_t xbuf;     // shared::cta address of this CTA's [2][kLnPeerSlots][128] double2
  uint32_t xfull;    // shared::cta address of this CTA's two exchange mbarriers
  int* err;
  volatile int* abort_flag;
};

// Fused residual + LayerNorm (model.go:743-769) over the BN-column slice
// [n0, n0 + BN) of a row whose full length is N: v = acc + bias + resid (the
// residual tile is already in shared memory) is written back to TMEM while
// Σv and Σv² accumulate in f64; the kParts warps of a lane quarter (one per
// column share) combine their sums through shared memory, the CTAs holding
// the row's other slices add theirs through distributed shared memory (in
// rank order, so every slice normalises with bit-identical statistics), then
// y = (v − mean)·inv·γ + β leaves through the TMA sink. `rrow` is this row's
// line in residual sub-tile 0 (128-byte swizzled rows); `cols` holds the
// slice's bias, γ and β (shared memory, BN f32 each); `resid_done` is called
// once the residual has been read. Returns false if a peer's sums did not
// arrive in time.
// Residual chunk (32 bf16 of one row) from global memory; zeros past M.
__device__ __forceinline__ void resid_fetch(const uint16_t* p, bool ok, uint4 (&dst)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    dst[i] = ok ? reinterpret_cast<const uint4*>(p)[i] : make_uint4(0u, 0u, 0u, 0u);
}

template <int BN, int kParts, bool kSmemResid, bool F16, typename Sink, typename Done>
__device__ __forceinline__ bool epilogue_resid_ln(uint32_t taddr, int row, int row0, int M, int N,
                                                  int n0, int part, int quarter, int lane,
                                                  const EpiParams& ep, double2* red, Sink& sink,
                                                  uint32_t rrow, uint4 (&rg)[2][4],
                                                  uint32_t cols, Done&& resid_done,
                                                  const LnPeers& px, int it) {
  constexpr int kCols = BN / kParts, kChunks = kCols / 32;
  const bool row_ok = row < M;
  const int c0 = part * kCols;
  const int swz = lane & 7;  // row & 7 (rows of a quarter start at multiples of 32)
  // Σv, Σv²: f32 over each 32-column chunk (paired lanes), then f64.
  double s1 = 0.0, s2 = 0.0;
  uint32_t ub[2][32];  // chunk k + 1's TMEM load is in flight while k is processed
  tmem_ld32(taddr + c0, ub[0]);
#pragma unroll
  for (int k = 0; k < kChunks; ++k) {
    const int c = c0 + 32 * k;
    uint32_t (&u)[32] = ub[k & 1];
    uint32_t w[16];  // 32 residual bf16
    if constexpr (kSmemResid) {
      const uint32_t sub = rrow + (uint32_t)(c / 64) * (128u * 128u);
      const int cc0 = (c % 64) / 8;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(w[4 * i]), "=r"(w[4 * i + 1]), "=r"(w[4 * i + 2]), "=r"(w[4 * i + 3])
                     : "r"(sub + (uint32_t)(((cc0 + i) ^ swz) << 4)));
    } else {
      // Chunks k and k + 1 were fetched ahead; fetch k + 2 into k's buffer.
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        w[4 * i] = rg[k & 1][i].x;
        w[4 * i + 1] = rg[k & 1][i].y;
        w[4 * i + 2] = rg[k & 1][i].z;
        w[4 * i + 3] = rg[k & 1][i].w;
      }
      if (k + 2 < kChunks)
        resid_fetch(reinterpret_cast<const uint16_t*>(ep.resid) + (size_t)row * ep.ldr + n0 +
                        c + 64,
                    row_ok, rg[k & 1]);
    }
    tmem_ld_wait();
    if (k + 1 < kChunks) {
      if (k > 0) tmem_st_wait();  // that buffer was chunk k − 1's store source
      tmem_ld32(taddr + c + 32, ub[(k + 1) & 1]);
    }
    uint64_t a1 = 0, a2 = 0;  // (0.f, 0.f)
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 bq = ld_shared_f4(cols + (uint32_t)(c + 4 * q) * 4u);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i = 2 * q + h;
        float rlo, rhi;
        unpack2_16<F16>(w[i], rlo, rhi);
        const uint64_t r2 = f2_pack(rlo, rhi);
        uint64_t v2 = f2_pack(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1]));
        v2 = f2_add(v2, h ? f2_pack(bq.z, bq.w) : f2_pack(bq.x, bq.y));
        v2 = f2_add(v2, r2);
        a1 = f2_add(a1, v2);
        a2 = f2_fma(v2, v2, a2);
        float x, y;
        f2_unpack(v2, x, y);
        u[2 * i] = __float_as_uint(x);
        u[2 * i + 1] = __float_as_uint(y);
      }
    }
    float p0, p1, q0, q1;
    f2_unpack(a1, p0, p1);
    f2_unpack(a2, q0, q1);
    s1 += (double)p0 + (double)p1;
    s2 += (double)q0 + (double)q1;
    tmem_st32(taddr + c, u);
  }
  resid_done();
  tmem_st_wait();
  const int slot = quarter * 32 + lane;
  double2* rp = red + (size_t)(it & 1) * kParts * 128;  // this tile's parity
  rp[part * 128 + slot] = make_double2(s1, s2);
  named_bar_sync(1 + quarter, 32 * kParts);
  // This slice's sums, added in part order: identical in every warp of the
  // quarter.
  double t1 = 0.0, t2 = 0.0;
#pragma unroll
  for (int q = 0; q < kParts; ++q) {
    const double2 o = rp[q * 128 + slot];
    t1 += o.x;
    t2 += o.y;
  }
  if (px.peers > 1) {
    const uint32_t par = (uint32_t)(it & 1);
    const uint32_t cell = px.xbuf + ((par * kLnPeerSlots + px.rank) * 128 + slot) * 16;
    // This tile's phase of the exchange barrier completes on one local
    // arrival that announces the bytes the peers send (16 per row and peer;
    // their stores may land before or after it).
    if (part == 0 && quarter == 0 && lane == 0)
      mbar_arrive_expect_tx(px.xfull + 8 * par, 128u * 16u * (uint32_t)(px.peers - 1));
    if (part == 0) {
      for (int r = 0; r < px.peers; ++r) {
        if (r == (int)px.rank) continue;
        const uint32_t cr = (uint32_t)r * px.rstride + px.rhalf;
        st_async_f64x2(mapa_shared(cell, cr), t1, t2, mapa_shared(px.xfull + 8 * par, cr));
      }
    }
    if (!mbar_wait_cluster_bounded(px.xfull + 8 * par, (uint32_t)(it >> 1) & 1u, px.err,
                                   kDevTimeoutLnPeer, px.abort_flag))
      return false;
    double a1 = 0.0, a2 = 0.0;
    const double2* xb = reinterpret_cast<const double2*>(__cvta_shared_to_generic(px.xbuf)) +
                        (size_t)par * kLnPeerSlots * 128 + slot;
    for (int r = 0; r < px.peers; ++r) {
      const double2 q = r == (int)px.rank ? make_double2(t1, t2) : xb[r * 128];
      a1 += q.x;
      a2 += q.y;
    }
    t1 = a1;
    t2 = a2;
  }
  const double mean = t1 / (double)N;
  double var = t2 / (double)N - mean * mean;
  var = var > 0.0 ? var : 0.0;
  const float inv = (float)(1.0 / sqrt(var + (double)ep.eps));
  const float mf = (float)mean;
  const uint64_t nm2 = f2_pack(-mf, -mf), inv2 = f2_pack(inv, inv);
  tmem_ld32(taddr + c0, ub[0]);
#pragma unroll
  for (int k = 0; k < kChunks; ++k) {
    const int c = c0 + 32 * k;
    const uint32_t (&u)[32] = ub[k & 1];
    tmem_ld_wait();
    if (k + 1 < kChunks) tmem_ld32(taddr + c + 32, ub[(k + 1) & 1]);
    float y[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 gq = ld_shared_f4(cols + (uint32_t)(BN + c + 4 * q) * 4u);
      const float4 eq = ld_shared_f4(cols + (uint32_t)(2 * BN + c + 4 * q) * 4u);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i = 2 * q + h;
        // ((v − mean)·inv)·γ + β, two columns per instruction.
        uint64_t t =
            f2_add(f2_pack(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1])), nm2);
        t = f2_mul(t, inv2);
        t = f2_fma(t, h ? f2_pack(gq.z, gq.w) : f2_pack(gq.x, gq.y),
                   h ? f2_pack(eq.z, eq.w) : f2_pack(eq.x, eq.y));
        f2_unpack(t, y[2 * i], y[2 * i + 1]);
      }
    }
    sink.put(y, n0 + c, row0);
    if (row_ok && ep.out_f32) store32<float>(ep.out_f32 + (size_t)row * N + n0 + c, y);
  }
  return true;
}

template <int BN, int EPI, bool S8, typename OutT, bool F16 = false, bool PAIR = false>
__global__ void __launch_bounds__(64 + 32 * gemm_epi_warps<BN, EPI, S8>(), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR,
                   int M, int N, int K, EpiParams ep, int* err) {
  // LayerNorm over rows wider than one tile: the grid is made of clusters of
  // N / BN column slices (CTA pairs with PAIR), the CTAs of slice r compute
  // columns [r·BN, r·BN + BN) of every row tile the cluster takes, and the
  // slices exchange row statistics. The producer loads each tile's residual
  // slice (tmR) next to the operands.
  constexpr bool kLnSlices = EPI == kEpiResidLN || EPI == kEpiResidLNG;
  constexpr bool kResidTma = EPI == kEpiResidLN;  // residual tile via TMA into shared memory
  static_assert(!kLnSlices || ((BN == 128 || BN == 192) && !S8),
                "LayerNorm slices are 128 or 192 bf16 columns");
  using C = GemmCfg<BN, S8, kLnSlices, gemm_epi_warps<BN, EPI, S8>(), kResidTma, PAIR>;
  // bf16 outputs leave through TMA tile stores; f32 outputs store directly.
  constexpr bool kTmaStore = sizeof(OutT) == 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* full_bar = bars;                       // [kStages] TMA → MMA
  uint64_t* empty_bar = bars + C::kStages;         // [kStages] MMA → TMA
  uint64_t* accf_bar = bars + 2 * C::kStages;      // [kNumAcc] MMA → epilogue
  uint64_t* acce_bar = accf_bar + 2;               // [kNumAcc] epilogue → MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* xfull_bar = acce_bar + 3;              // [2] peers → LayerNorm epilogue
  uint64_t* rfull_bar = acce_bar + 5;              // residual tile: TMA → epilogue
  uint64_t* rempty_bar = acce_bar + 6;             // residual tile: epilogue → TMA
  // Extra region: LayerNorm kernels keep their partial sums (kRedBytes),
  // then one 2 KB staging buffer per epilogue warp; other kernels two per warp.
  uint8_t* extra = smem + C::kExtraOffset;
  double2* red = reinterpret_cast<double2*>(extra);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + C::kTileM - 1) / C::kTileM;
  const int num_n = (N + BN - 1) / BN;
  const int num_k = (K + C::kBK - 1) / C::kBK;
  // Cluster layout: rank = slice · (PAIR ? 2 : 1) + half. With PAIR the even
  // CTA of a pair (the leader) issues the pair's MMAs, waits for both CTAs'
  // operand bytes on its full barriers and for both CTAs' epilogues on its
  // accumulator-empty barriers; commits arrive in both CTAs.
  const uint32_t crank = (kLnSlices || PAIR) ? cluster_ctarank() : 0u;
  const uint32_t half = PAIR ? (crank & 1u) : 0u;
  const uint32_t leader = crank & ~1u;  // the pair's even rank (PAIR)
  const bool is_leader = !PAIR || half == 0;
  const uint16_t pair_mask = (uint16_t)(3u << leader);
  // Tile loop: tiles first, first + stride, ... < num_tiles; tile → (mb, nb).
  const int peers = kLnSlices ? num_n : 1;
  const int csize = peers * (PAIR ? 2 : 1);  // CTAs per cluster
  const uint32_t rank = PAIR ? crank >> 1 : crank;  // this CTA's column slice (kLnSlices)
  const int num_tiles = kLnSlices ? num_m : num_m * num_n;
  const int first = (int)blockIdx.x / csize;
  const int stride = (int)gridDim.x / csize;
  auto tile_mb = [&](int t) { return kLnSlices ? t : t / num_n; };
  auto tile_nb = [&](int t) { return kLnSlices ? (int)rank : t % num_n; };
  // This CTA's first row of a tile's rows.
  auto tile_row0 = [&](int mb) { return mb * C::kTileM + (int)half * C::kBM; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&accf_bar[a]), 1);
      // One arrive per epilogue warp (of both CTAs of a pair).
      mbar_init(smem_u32(&acce_bar[a]), (PAIR ? 2 : 1) * C::kEpiWarps);
      // One local arrival per tile, plus the peers' asynchronous stores
      // counted in bytes (epilogue_resid_ln).
      if (kLnSlices) mbar_init(smem_u32(&xfull_bar[a]), 1u);
    }
    if (kResidTma) {
      mbar_init(smem_u32(rfull_bar), 1);
      mbar_init(smem_u32(rempty_bar), C::kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    if constexpr (kTmaStore) tma_prefetch_desc(&tmO);
    if constexpr (kResidTma) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_u32(tmem_slot), C::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
      tmem_relinquish();
    }
  }
  if constexpr (kLnSlices) {
    // The slice's bias, γ and β, read by every tile's epilogue.
    float* cs = reinterpret_cast<float*>(smem + C::kColsOffset);
    const int n0 = (int)rank * BN;
    for (int i = threadIdx.x; i < BN; i += blockDim.x) {
      cs[i] = ep.bias ? ep.bias[n0 + i] : 0.0f;
      cs[BN + i] = ep.ln_w[n0 + i];
      cs[2 * BN + i] = ep.ln_b[n0 + i];
    }
  }
  tc_fence_before();
  // Peers' barriers exist before any remote arrive.
  if constexpr (kLnSlices || PAIR) cluster_sync_all();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Activations and outputs only after the previous kernel has completed.
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0, rtiles = 0;
      // The residual slice of a tile is loaded once the epilogue has read the
      // previous tile's, after the tile's first ring-full of k-blocks: those
      // loads go out while the previous tile's epilogue still holds the
      // residual buffer, so the MMAs of this tile start on time.
      const int resid_after = (num_k < C::kStages ? num_k : C::kStages) - 1;
      for (int tile = first; tile < num_tiles; tile += stride) {
        const int mb = tile_mb(tile), nb = tile_nb(tile);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&empty_bar[stage]), phase ^ 1u, err, kDevTimeoutSmemEmpty,
                                 abort_flag))
            goto producer_done;
          uint8_t* sa = smem + stage * C::kStageBytes;
          uint8_t* sb = sa + C::kABytes;
          const uint32_t fb = smem_u32(&full_bar[stage]);
          if constexpr (PAIR) {
            // Both CTAs' bytes complete the leader's barrier; the leader
            // announces them (a peer's bytes may land first: the phase cannot
            // complete before the leader's arrival).
            if (is_leader) mbar_arrive_expect_tx(fb, 2 * C::kStageBytes);
            const uint32_t cfb = mapa_shared(fb, leader);
            tma_load_2d_pair(smem_u32(sa), &tmA, cfb, kb * C::kBK, tile_row0(mb));
            tma_load_2d_pair(smem_u32(sb), &tmW, cfb, kb * C::kBK, nb * BN + (int)half * C::kBRows);
          } else {
            mbar_arrive_expect_tx(fb, C::kStageBytes);
            tma_load_2d(smem_u32(sa), &tmA, fb, kb * C::kBK, mb * C::kBM);
            tma_load_2d(smem_u32(sb), &tmW, fb, kb * C::kBK, nb * BN);
          }
          ++issued;
          if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
          if constexpr (kResidTma) {
            if (kb == resid_after) {
              if (!mbar_wait_bounded(smem_u32(rempty_bar), ((uint32_t)rtiles & 1u) ^ 1u, err,
                                     kDevTimeoutSmemEmpty, abort_flag))
                goto producer_done;
              const uint32_t rb = smem_u32(rfull_bar);
              mbar_arrive_expect_tx(rb, C::kResidBytes);
#pragma unroll
              for (int g = 0; g < BN / 64; ++g)
                tma_load_2d(smem_u32(smem + C::kResidOffset + g * C::kBM * 128), &tmR, rb,
                            nb * BN + g * 64, tile_row0(mb));
              ++rtiles;
            }
          }
        }
      }
    producer_done:
      // Drain: make sure this thread's own copies have landed before exit.
      if (kResidTma && rtiles > 0) {
        uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(smem_u32(rfull_bar), (uint32_t)(rtiles - 1) & 1u)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) break;
        }
      }
      // A pair's operand bytes all complete the leader's full barriers, so the
      // leader drains for both (the peer cannot leave before it: the kernel
      // ends with a cluster barrier).
      if (is_leader) {
        int n = issued < C::kStages ? issued : C::kStages;
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < n; ++i) {
          if (--s < 0) { s = C::kStages - 1; ph ^= 1u; }
          uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(smem_u32(&full_bar[s]), ph)) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && is_leader) {
      // ---------------- MMA issuer ----------------
      // Operand format: S8 (kind::i8), else F16 = 0 / BF16 = 1 (kind::f16).
      constexpr uint32_t idesc = make_idesc(S8 ? 2u : 1u, (S8 || !F16) ? 1u : 0u,
                                            (uint32_t)C::kTileM, (uint32_t)C::kMmaN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int tile = first; tile < num_tiles; tile += stride, ++it) {
        const int acc = it % C::kNumAcc;
        const uint32_t acc_phase = (uint32_t)(it / C::kNumAcc) & 1u;
        // A pair's accumulator is free once both CTAs' epilogues have read it.
        const bool freed =
            PAIR ? mbar_wait_cluster_bounded(smem_u32(&acce_bar[acc]), acc_phase ^ 1u, err,
                                             kDevTimeoutAccEmpty, abort_flag)
                 : mbar_wait_bounded(smem_u32(&acce_bar[acc]), acc_phase ^ 1u, err,
                                     kDevTimeoutAccEmpty, abort_flag);
        if (!freed) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::kAccStride;
        bool ok = true;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&full_bar[stage]), phase, err, kDevTimeoutTmaFull,
                                 abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* sa = smem + stage * C::kStageBytes;
          const uint64_t adesc = smem_desc_k_sw128(smem_u32(sa));
          const uint64_t bdesc = smem_desc_k_sw128(smem_u32(sa + C::kABytes));
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            // +32 bytes along K inside the 128-byte swizzle row (encoded >> 4).
            const uint64_t koff = (uint64_t)(ks * 2);
            if constexpr (S8)
              mma_s8(d_tmem, adesc + koff, bdesc + koff, idesc, (kb | ks) ? 1u : 0u);
            else if constexpr (PAIR)
              mma_f16kind_pair(d_tmem, adesc + koff, bdesc + koff, idesc, (kb | ks) ? 1u : 0u);
            else
              mma_f16kind(d_tmem, adesc + koff, bdesc + koff, idesc, (kb | ks) ? 1u : 0u);
          }
          if constexpr (PAIR) mma_commit_pair(smem_u32(&empty_bar[stage]), pair_mask);
          else mma_commit(smem_u32(&empty_bar[stage]));
          if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
        }
        if constexpr (PAIR) mma_commit_pair(smem_u32(&accf_bar[acc]), pair_mask);
        else mma_commit(smem_u32(&accf_bar[acc]));
        if (!ok) break;
      }
      // Drain: wait (bounded) for the last committed MMAs before TMEM is freed.
      if (it > 0) {
        const int acc = (it - 1) % C::kNumAcc;
        const uint32_t acc_phase = (uint32_t)((it - 1) / C::kNumAcc) & 1u;
        uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(smem_u32(&accf_bar[acc]), acc_phase)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) break;
        }
      }
    }
  } else {
    // ---------------- epilogue warps 2..9 ----------------
    const int quarter = warp & 3;        // TMEM lanes [32*quarter, 32*quarter+32)
    const int part = (warp - 2) >> 2;    // which share of the column chunks
    TmaSink<2> tsink{extra + (warp - 2) * 4096, &tmO, lane, 0, F16 ? 0 : ep.f16_from};
    TmaSink<1> lsink{extra + C::kRedBytes + (warp - 2) * 2048, &tmO, lane, 0, F16 ? 0 : 1 << 30};
    const LnPeers px{peers, rank, PAIR ? 2u : 1u, half, smem_u32(smem + C::kXchOffset),
                     smem_u32(xfull_bar), err, abort_flag};
    // The accumulator-empty barrier this CTA's epilogue arrives on: its own,
    // or the pair leader's.
    const uint32_t acce_dst = PAIR ? mapa_shared(smem_u32(acce_bar), leader) : smem_u32(acce_bar);
    int it = 0;
    for (int tile = first; tile < num_tiles; tile += stride, ++it) {
      const int acc = it % C::kNumAcc;
      const uint32_t acc_phase = (uint32_t)(it / C::kNumAcc) & 1u;
      const int mb = tile_mb(tile), nb = tile_nb(tile);
      const int row0 = tile_row0(mb) + quarter * 32;
      const int row = row0 + lane;
      // Global-residual LayerNorm: the first two chunks are fetched while the
      // tile's MMAs finish.
      uint4 rg[2][4];
      if constexpr (kLnSlices && !kResidTma) {
        const uint16_t* rp = reinterpret_cast<const uint16_t*>(ep.resid) +
                             (size_t)row * ep.ldr + nb * BN + part * (BN / C::kParts);
        resid_fetch(rp, row < M, rg[0]);
        resid_fetch(rp + 32, row < M, rg[1]);
      }
      if (!mbar_wait_bounded(smem_u32(&accf_bar[acc]), acc_phase, err, kDevTimeoutAccFull,
                             abort_flag))
        break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + acc * C::kAccStride + ((uint32_t)(quarter * 32) << 16);
      if constexpr (kLnSlices) {
        if (kResidTma && !mbar_wait_bounded(smem_u32(rfull_bar), (uint32_t)it & 1u, err,
                                            kDevTimeoutTmaFull, abort_flag))
          break;
        const uint32_t rrow = smem_u32(smem + C::kResidOffset) + (uint32_t)(quarter * 32 + lane) * 128u;
        auto resid_done = [&]() {
          if constexpr (kResidTma) {
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(rempty_bar));
          }
        };
        if (!epilogue_resid_ln<BN, C::kParts, kResidTma, F16>(
                taddr, row, row0, M, N, nb * BN, part, quarter, lane, ep, red, lsink, rrow, rg,
                smem_u32(smem + C::kColsOffset), resid_done, px, it))
          break;
      } else if constexpr (kTmaStore) {
        epilogue_row<BN, EPI, S8, C::kParts>(taddr, row, row0, M, N, nb, part, ep, tsink);
      } else {
        DirectSink<OutT> dsink{reinterpret_cast<OutT*>(ep.out), ep.ldo, row, row < M,
                               EPI == kEpiSwiglu ? N / 2 : N};
        epilogue_row<BN, EPI, S8, C::kParts>(taddr, row, row0, M, N, nb, part, ep, dsink);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) mbar_arrive_cluster(acce_dst + 8u * (uint32_t)acc);
        else mbar_arrive(acce_dst + 8u * (uint32_t)acc);
      }
    }
    // The last tile's TMA stores read their staging before the CTA exits.
    if constexpr (kLnSlices) lsink.drain();
    else if constexpr (kTmaStore) tsink.drain();
  }

  __syncthreads();
  // No CTA of a cluster leaves while a peer may still store into its shared
  // memory or issue MMAs into its TMEM (every wait above is bounded, so all
  // CTAs get here).
  if constexpr (kLnSlices || PAIR) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C::kTmemCols);
    else tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

}  // namespace futon
