// gemm_launch.cuh — host-side launch of the tcgen05 GEMM instantiations.
#pragma once

#include <atomic>

#include "gemm_tc.cuh"

namespace futon {

struct GemmLaunch {
  const CUtensorMap* ta;  // A [M, K] (bf16 or s8), box 128 × 128 bytes
  const CUtensorMap* tw;  // W [N, K], box bn × 128 bytes
  const CUtensorMap* to;  // bf16 output [M, ncols], box 32 × 32, 64B swizzle (TMA-store epilogues)
  const CUtensorMap* tr;  // kEpiResidLN: bf16 residual [M, N], box 64 × 128, 128B swizzle
  int M, N, K;
  int bn;                 // 64, 128, 192 or 256
  int epi;                // EpiKind
  bool out_f32;           // output element type: f32 (true) or 16-bit (bf16, or f16 with f16)
  bool f16;               // 16-bit operands, outputs and residuals are f16 (else bf16)
  bool pair;              // f16 only: CTA-pair tiles (M = 256, cta_group::2); tw's box is bn / 2 rows
  bool pdl;               // programmatic dependent launch (the kernel waits with griddepcontrol.wait)
  EpiParams ep;
  int* err;               // device error word
  int num_sms;
  cudaStream_t stream;
};

// Defined in gemm_f16.cu (the forward's f16 GEMMs, every epilogue),
// gemm_bf16.cu (the MatMulT seam: bf16 operands, f32 output, bias only) and
// gemm_s8.cu (the int8 path).
cudaError_t launch_gemm_f16(const GemmLaunch& g);
cudaError_t launch_gemm_bf16(const GemmLaunch& g);
cudaError_t launch_gemm_s8(const GemmLaunch& g);

template <int BN, int EPI, bool S8, typename OutT, bool F16, bool PAIR>
cudaError_t launch_gemm_inst_p(const GemmLaunch& g) {
  constexpr bool kLn = EPI == kEpiResidLN || EPI == kEpiResidLNG;
  using C = GemmCfg<BN, S8, kLn, gemm_epi_warps<BN, EPI, S8>(), EPI == kEpiResidLN, PAIR>;
  auto kern = gemm_tc_kernel<BN, EPI, S8, OutT, F16, PAIR>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<uint64_t> attr_done{0};  // one bit per device
  if (!(attr_done.load() & (1ull << (dev & 63)))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(1ull << (dev & 63));
  }
  constexpr bool kTmaStore = sizeof(OutT) == 2;
  if (kTmaStore && !g.to) return cudaErrorInvalidValue;  // bf16 outputs need an output map
  const long num_m = (g.M + C::kTileM - 1) / C::kTileM;
  if (num_m == 0) return cudaSuccess;
  if constexpr (kLn) {
    // N / BN column slices of a row tile per cluster.
    if (g.N % BN != 0 || g.N / BN < 2 || g.N / BN > kLnPeerSlots || !g.tr)
      return cudaErrorInvalidValue;
  }
  const int peers = kLn ? g.N / BN : 1;
  const int csize = peers * (PAIR ? 2 : 1);  // CTAs per cluster
  const long tiles = kLn ? num_m : num_m * ((g.N + BN - 1) / BN);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (csize > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)csize;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (g.pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = g.stream;
  cfg.attrs = na ? attr : nullptr;
  cfg.numAttrs = (unsigned)na;
  if (csize == 1) {
    cfg.gridDim = dim3((unsigned)(tiles < g.num_sms ? tiles : g.num_sms));
    return cudaLaunchKernelEx(&cfg, kern, *g.ta, *g.tw, g.to ? *g.to : *g.ta, *g.ta, g.M, g.N, g.K,
                              g.ep, g.err);
  }
  // Clusters that fit at once (per device and cluster size, queried once).
  static std::atomic<int> fit_cache[64][2 * kLnPeerSlots + 1];
  int fit = fit_cache[dev & 63][csize].load();
  if (fit == 0) {
    cfg.gridDim = dim3((unsigned)(csize * (g.num_sms / csize)));
    cudaError_t e = cudaOccupancyMaxActiveClusters(&fit, kern, &cfg);
    if (e != cudaSuccess) return e;
    if (fit <= 0) return cudaErrorInvalidConfiguration;
    fit_cache[dev & 63][csize].store(fit);
  }
  const int clusters = (int)(tiles < fit ? tiles : fit);
  cfg.gridDim = dim3((unsigned)(clusters * csize));
  return cudaLaunchKernelEx(&cfg, kern, *g.ta, *g.tw, g.to ? *g.to : *g.ta, g.tr ? *g.tr : *g.ta,
                            g.M, g.N, g.K, g.ep, g.err);
}

// The CTA-pair form for the f16 forward (g.pair), else one CTA per tile.
template <int BN, int EPI, bool S8, typename OutT, bool F16 = false>
cudaError_t launch_gemm_inst(const GemmLaunch& g) {
  if constexpr (F16 && !S8) {
    if (g.pair) return launch_gemm_inst_p<BN, EPI, S8, OutT, F16, true>(g);
  } else {
    if (g.pair) return cudaErrorInvalidValue;
  }
  return launch_gemm_inst_p<BN, EPI, S8, OutT, F16, false>(g);
}

template <bool S8, int BN, bool F16>
cudaError_t launch_gemm_bn(const GemmLaunch& g) {
  using H = __half;
  if constexpr (!S8 && F16) {
    switch (g.epi) {
      case kEpiStore:
        return g.out_f32 ? launch_gemm_inst<BN, kEpiStore, false, float, true>(g)
                         : launch_gemm_inst<BN, kEpiStore, false, H, true>(g);
      case kEpiRope:
        return g.out_f32 ? launch_gemm_inst<BN, kEpiRope, false, float, true>(g)
                         : launch_gemm_inst<BN, kEpiRope, false, H, true>(g);
      case kEpiGelu: return launch_gemm_inst<BN, kEpiGelu, false, H, true>(g);
      case kEpiSwiglu:
        if constexpr (BN != 192) return launch_gemm_inst<BN, kEpiSwiglu, false, H, true>(g);
        else return cudaErrorInvalidValue;
      case kEpiResid: return launch_gemm_inst<BN, kEpiResid, false, float, true>(g);
      case kEpiResidLN:
        // Long-K GEMMs (fc2) take the global-residual variant and its extra
        // pipeline stage; short ones (out) the TMA-loaded residual tile.
        if constexpr (BN == 128 || BN == 192)
          return g.K >= 1024 ? launch_gemm_inst<BN, kEpiResidLNG, false, H, true>(g)
                             : launch_gemm_inst<BN, kEpiResidLN, false, H, true>(g);
        else return cudaErrorInvalidValue;
    }
  } else if constexpr (!S8) {
    // The MatMulT seam: f32 output, bias only.
    if (g.epi == kEpiStore && g.out_f32) return launch_gemm_inst<BN, kEpiStore, false, float>(g);
  } else {
    switch (g.epi) {
      case kEpiStore:
        return g.out_f32 ? launch_gemm_inst<BN, kEpiStore, true, float>(g)
                         : launch_gemm_inst<BN, kEpiStore, true, __nv_bfloat16>(g);
      case kEpiRope:
        return g.out_f32 ? launch_gemm_inst<BN, kEpiRope, true, float>(g)
                         : launch_gemm_inst<BN, kEpiRope, true, __nv_bfloat16>(g);
      case kEpiGelu: return launch_gemm_inst<BN, kEpiGelu, true, float>(g);
      case kEpiSwiglu:
        if constexpr (BN != 192) return launch_gemm_inst<BN, kEpiSwiglu, true, float>(g);
        else return cudaErrorInvalidValue;
      case kEpiResid: return launch_gemm_inst<BN, kEpiResid, true, float>(g);
    }
  }
  return cudaErrorInvalidValue;
}

template <bool S8, bool F16>
cudaError_t launch_gemm_any(const GemmLaunch& g) {
  switch (g.bn) {
    case 64: return launch_gemm_bn<S8, 64, F16>(g);
    case 128: return launch_gemm_bn<S8, 128, F16>(g);
    case 192: return launch_gemm_bn<S8, 192, F16>(g);
    case 256: return launch_gemm_bn<S8, 256, F16>(g);
  }
  return cudaErrorInvalidValue;
}

}  // namespace futon
