// rowops.cuh — HBM-bound row kernels of the encoder forward.
//
//   embed_ln_kernel   word[id] + type[0] + pos[t], then LayerNorm
//                     (model.go:384-396) — warp per token
//   layernorm_kernel  LayerNorm of the residual sum the out/fc2 GEMM
//                     epilogue wrote (model.go:597-599, 631-633)
//   quant_rows_kernel per-row symmetric int8 quantisation (quant.go:42-70)
//   pool_kernel       CLS / mean pooling, matryoshka LayerNorm, L2
//                     (model.go:416-453) — one CTA per sequence
//   gather_rows_kernel CLS rows of the residual stream for the pruned last
//                     layer (model.go:403-410)
//
// LayerNorm statistics follow layerNormRows (model.go:743-769): mean and
// variance accumulate in float64, inv = float32(1/sqrt(var + eps)), and the
// apply step (x − mean)·inv·γ + β runs as separately rounded f32 ops.
// Each LayerNorm writes the f32 row (the residual for the next block), its
// f16 copy (the next GEMM's A operand) and, on the int8 path, the row's
// int8 codes and scale.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "mathf32.cuh"

namespace futon {

constexpr int kMaxRowVec = 8;  // float4 per lane → hidden ≤ 1024

// Quantises one row held as float4 registers across a warp (quant.go:42-70):
// scale = amax/127 (f32), codes = round-half-away(v · (127/amax)) in f64,
// clamped to ±127; an all-zero row gets scale 0 and zero codes.
__device__ __forceinline__ void warp_quant_row(const float4 (&v)[kMaxRowVec], int n4, int lane,
                                               int8_t* q, float* scale_out) {
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxRowVec; ++j) {
    const int c4 = lane + 32 * j;
    if (c4 < n4) {
      amax = fmaxf(amax, fabsf(v[j].x));
      amax = fmaxf(amax, fabsf(v[j].y));
      amax = fmaxf(amax, fabsf(v[j].z));
      amax = fmaxf(amax, fabsf(v[j].w));
    }
  }
  amax = warp_max(amax);
  const double inv = amax == 0.f ? 0.0 : 127.0 / (double)amax;
#pragma unroll
  for (int j = 0; j < kMaxRowVec; ++j) {
    const int c4 = lane + 32 * j;
    if (c4 < n4) {
      float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
      char4 out;
      int8_t* o = reinterpret_cast<int8_t*>(&out);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        double r = round((double)e[t] * inv);
        r = fmin(127.0, fmax(-127.0, r));
        o[t] = (int8_t)r;
      }
      reinterpret_cast<char4*>(q)[c4] = out;
    }
  }
  if (lane == 0) *scale_out = amax == 0.f ? 0.f : __fdiv_rn(amax, 127.0f);
}

// Row statistics in layerNormRows' exact order (model.go:743-769): one
// lane sums the row (staged in this warp's shared-memory row `srow`) in
// element order in float64, mean = Σx / h, then Σ (x − mean)² with every
// product and sum rounded separately, / h. For the int8 path's exact mode,
// whose per-row quantisation turns any float32 difference in a row's mean or
// 1/σ into whole code steps.
__device__ __forceinline__ void warp_row_stats_seq(const float4 (&v)[kMaxRowVec], int h, int lane,
                                                   float* srow, double* mean_out,
                                                   double* var_out) {
  const int n4 = h >> 2;
#pragma unroll
  for (int j = 0; j < kMaxRowVec; ++j)
    if (lane + 32 * j < n4) reinterpret_cast<float4*>(srow)[lane + 32 * j] = v[j];
  __syncwarp();
  double mean = 0.0, var = 0.0;
  if (lane == 0) {
    for (int i = 0; i < h; ++i) mean = __dadd_rn(mean, (double)srow[i]);
    mean = __ddiv_rn(mean, (double)h);
    for (int i = 0; i < h; ++i) {
      const double d = __dsub_rn((double)srow[i], mean);
      var = __dadd_rn(var, __dmul_rn(d, d));
    }
    var = __ddiv_rn(var, (double)h);
  }
  *mean_out = __shfl_sync(0xffffffffu, mean, 0);
  *var_out = __shfl_sync(0xffffffffu, var, 0);
  __syncwarp();  // srow is free for the warp's next row
}

// Two f32 values as an f16x2 word (low half first), saturating at ±65504.
__device__ __forceinline__ uint32_t pack2_f16_sat(float lo, float hi) {
  uint32_t w;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(w) : "f"(hi), "f"(lo));
  return w;
}

__device__ __forceinline__ void warp_layernorm_apply(float4 (&v)[kMaxRowVec], int h, int lane,
                                                     const float* __restrict__ w,
                                                     const float* __restrict__ b, float eps,
                                                     double mean, double var,
                                                     float* __restrict__ xo,
                                                     __half* __restrict__ xbo,
                                                     int8_t* __restrict__ xq,
                                                     float* __restrict__ xs);

// LayerNorm of a row held as float4 registers; writes f32, f16 and
// optionally int8 outputs. SEQ: statistics by warp_row_stats_seq (srow: this
// warp's h floats of shared memory); otherwise a warp-parallel float64 sum.
template <bool SEQ = false>
__device__ __forceinline__ void warp_layernorm_store(float4 (&v)[kMaxRowVec], int h, int lane,
                                                     const float* __restrict__ w,
                                                     const float* __restrict__ b, float eps,
                                                     float* __restrict__ xo,
                                                     __half* __restrict__ xbo,
                                                     int8_t* __restrict__ xq,
                                                     float* __restrict__ xs,
                                                     float* srow = nullptr) {
  const int n4 = h >> 2;
  double mean, var;
  if constexpr (SEQ) {
    warp_row_stats_seq(v, h, lane, srow, &mean, &var);
  } else {
    double sum = 0.0;
#pragma unroll
    for (int j = 0; j < kMaxRowVec; ++j)
      if (lane + 32 * j < n4)
        sum += ((double)v[j].x + (double)v[j].y) + ((double)v[j].z + (double)v[j].w);
    mean = warp_sum_d(sum) / (double)h;
    var = 0.0;
#pragma unroll
    for (int j = 0; j < kMaxRowVec; ++j) {
      if (lane + 32 * j < n4) {
        double a = (double)v[j].x - mean, bb = (double)v[j].y - mean;
        double c = (double)v[j].z - mean, d = (double)v[j].w - mean;
        var += (a * a + bb * bb) + (c * c + d * d);
      }
    }
    var = warp_sum_d(var) / (double)h;
  }
  warp_layernorm_apply(v, h, lane, w, b, eps, mean, var, xo, xbo, xq, xs);
}

// Row statistics of 32 rows at once in layerNormRows' exact order
// (model.go:743-769): lane l takes row x + l·h (rows past `n` give 0) and
// sums it in element order in float64 — mean = Σx / h, then Σ (x − mean)²
// with every product and sum rounded separately, / h — the same operations,
// in the same order, as warp_row_stats_seq, one row per lane.
__device__ __forceinline__ void warp_rows_stats_seq32(const float* __restrict__ x, int n, int h,
                                                      int lane, double* mean_out,
                                                      double* var_out) {
  double mean = 0.0, var = 0.0;
  if (lane < n) {
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)lane * h);
    const int n4 = h >> 2;
    for (int c = 0; c < n4; ++c) {
      const float4 a = xr[c];
      mean = __dadd_rn(mean, (double)a.x);
      mean = __dadd_rn(mean, (double)a.y);
      mean = __dadd_rn(mean, (double)a.z);
      mean = __dadd_rn(mean, (double)a.w);
    }
    mean = __ddiv_rn(mean, (double)h);
    for (int c = 0; c < n4; ++c) {
      const float4 a = xr[c];
      const float e[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const double d = __dsub_rn((double)e[t], mean);
        var = __dadd_rn(var, __dmul_rn(d, d));
      }
    }
    var = __ddiv_rn(var, (double)h);
  }
  *mean_out = mean;
  *var_out = var;
}

// The apply step of a LayerNorm whose statistics are known:
// y = (x − mean)·inv·γ + β with inv = float32(1/sqrt(var + eps)), then the
// f32 / f16 / int8 outputs.
__device__ __forceinline__ void warp_layernorm_apply(float4 (&v)[kMaxRowVec], int h, int lane,
                                                     const float* __restrict__ w,
                                                     const float* __restrict__ b, float eps,
                                                     double mean, double var,
                                                     float* __restrict__ xo,
                                                     __half* __restrict__ xbo,
                                                     int8_t* __restrict__ xq,
                                                     float* __restrict__ xs) {
  const int n4 = h >> 2;
  const float inv = (float)(1.0 / sqrt(var + (double)eps));
  const float mf = (float)mean;
#pragma unroll
  for (int j = 0; j < kMaxRowVec; ++j) {
    const int c4 = lane + 32 * j;
    if (c4 < n4) {
      const float4 g = reinterpret_cast<const float4*>(w)[c4];
      const float4 be = reinterpret_cast<const float4*>(b)[c4];
      float4 y;
      y.x = fadd(fmul(fmul(fsub(v[j].x, mf), inv), g.x), be.x);
      y.y = fadd(fmul(fmul(fsub(v[j].y, mf), inv), g.y), be.y);
      y.z = fadd(fmul(fmul(fsub(v[j].z, mf), inv), g.z), be.z);
      y.w = fadd(fmul(fmul(fsub(v[j].w, mf), inv), g.w), be.w);
      v[j] = y;
      if (xo) reinterpret_cast<float4*>(xo)[c4] = y;
      if (xbo)
        reinterpret_cast<uint2*>(xbo)[c4] = make_uint2(pack2_f16_sat(y.x, y.y),
                                                       pack2_f16_sat(y.z, y.w));
    }
  }
  if (xq) warp_quant_row(v, n4, lane, xq, xs);
}

// One warp per token row; each warp takes a contiguous run of tokens, so the
// sequence (for the position row) is found by one binary search per run and
// then advanced token by token.
// SEQ: LayerNorm statistics in the reference's exact order (int8 exact mode).
template <bool SEQ = false>
__global__ void __launch_bounds__(256)
    embed_ln_kernel(const int* __restrict__ ids, const int* __restrict__ cu, int nseq, int T,
                    int h, int vocab, int* __restrict__ err, const float* __restrict__ word, const float* __restrict__ type0,
                    const float* __restrict__ pos, const float* __restrict__ w,
                    const float* __restrict__ b, float eps, float* __restrict__ x,
                    __half* __restrict__ xb, int8_t* __restrict__ xq,
                    float* __restrict__ xs) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int n4 = h >> 2;
  const int per = (T + warps - 1) / warps;
  const int t0 = ((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * per;
  const int t1 = min(T, t0 + per);
  int s = 0;
  if (pos && t0 < t1) {
    int lo = 0, hi = nseq;  // cu[lo] ≤ t0 < cu[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (cu[mid] <= t0) lo = mid; else hi = mid;
    }
    s = lo;
  }
  for (int t = t0; t < t1; ++t) {
    int id = ids[t];
    if ((unsigned)id >= (unsigned)vocab) {  // device-resident ids are not host-checked
      if (lane == 0) atomicCAS(err, 0, (int)kDevBadInput);
      id = 0;
    }
    const float* wr = word + (size_t)id * h;
    const float* pr = nullptr;
    if (pos) {
      while (t >= cu[s + 1]) ++s;
      pr = pos + (size_t)(t - cu[s]) * h;
    }
    float4 v[kMaxRowVec];
#pragma unroll
    for (int j = 0; j < kMaxRowVec; ++j) {
      const int c4 = lane + 32 * j;
      if (c4 < n4) {
        float4 a = reinterpret_cast<const float4*>(wr)[c4];
        if (type0) {
          float4 tt = reinterpret_cast<const float4*>(type0)[c4];
          a.x = fadd(a.x, tt.x); a.y = fadd(a.y, tt.y); a.z = fadd(a.z, tt.z); a.w = fadd(a.w, tt.w);
        }
        if (pr) {
          float4 pp = reinterpret_cast<const float4*>(pr)[c4];
          a.x = fadd(a.x, pp.x); a.y = fadd(a.y, pp.y); a.z = fadd(a.z, pp.z); a.w = fadd(a.w, pp.w);
        }
        v[j] = a;
      } else {
        v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if constexpr (SEQ) {
      __shared__ __align__(16) float srows[8][kMaxRowVec * 128];
      warp_layernorm_store<true>(v, h, lane, w, b, eps, x ? x + (size_t)t * h : nullptr,
                                 xb ? xb + (size_t)t * h : nullptr,
                                 xq ? xq + (size_t)t * h : nullptr, xq ? xs + t : nullptr,
                                 srows[threadIdx.x >> 5]);
    } else {
      warp_layernorm_store(v, h, lane, w, b, eps, x ? x + (size_t)t * h : nullptr,
                           xb ? xb + (size_t)t * h : nullptr, xq ? xq + (size_t)t * h : nullptr,
                           xq ? xs + t : nullptr);
    }
  }
}

template <bool SEQ = false>
__global__ void __launch_bounds__(256)
    layernorm_kernel(const float* __restrict__ in, int rows, int h, const float* __restrict__ w,
                     const float* __restrict__ b, float eps, float* __restrict__ x,
                     __half* __restrict__ xb, int8_t* __restrict__ xq,
                     float* __restrict__ xs) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int n4 = h >> 2;
  if constexpr (SEQ) {
    // 32 rows per warp: each lane takes one row's statistics in the
    // reference's order, then the warp normalises the rows one by one.
    const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    for (int base = wid * 32; base < rows; base += warps * 32) {
      const int nr = min(32, rows - base);
      double mean, var;
      warp_rows_stats_seq32(in + (size_t)base * h, nr, h, lane, &mean, &var);
      for (int k = 0; k < nr; ++k) {
        const int r = base + k;
        const double mk = __shfl_sync(0xffffffffu, mean, k);
        const double vk = __shfl_sync(0xffffffffu, var, k);
        const float4* src = reinterpret_cast<const float4*>(in + (size_t)r * h);
        float4 v[kMaxRowVec];
#pragma unroll
        for (int j = 0; j < kMaxRowVec; ++j) {
          const int c4 = lane + 32 * j;
          v[j] = c4 < n4 ? src[c4] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        warp_layernorm_apply(v, h, lane, w, b, eps, mk, vk, x ? x + (size_t)r * h : nullptr,
                             xb ? xb + (size_t)r * h : nullptr, xq ? xq + (size_t)r * h : nullptr,
                             xq ? xs + r : nullptr);
      }
    }
  } else {
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
      const float4* src = reinterpret_cast<const float4*>(in + (size_t)r * h);
      float4 v[kMaxRowVec];
#pragma unroll
      for (int j = 0; j < kMaxRowVec; ++j) {
        const int c4 = lane + 32 * j;
        v[j] = c4 < n4 ? src[c4] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      warp_layernorm_store(v, h, lane, w, b, eps, x ? x + (size_t)r * h : nullptr,
                           xb ? xb + (size_t)r * h : nullptr, xq ? xq + (size_t)r * h : nullptr,
                           xq ? xs + r : nullptr);
    }
  }
}

// Per-row int8 quantisation of an f32 [rows, k] matrix (k % 4 == 0), warp
// per row, any k: pass 1 finds the absmax, pass 2 writes codes.
__global__ void __launch_bounds__(256)
    quant_rows_kernel(const float* __restrict__ in, int rows, int k, int8_t* __restrict__ q,
                      float* __restrict__ scale) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int n4 = k >> 2;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const float4* src = reinterpret_cast<const float4*>(in + (size_t)r * k);
    float amax = 0.f;
    for (int c4 = lane; c4 < n4; c4 += 32) {
      float4 a = src[c4];
      amax = fmaxf(fmaxf(amax, fabsf(a.x)), fmaxf(fabsf(a.y), fmaxf(fabsf(a.z), fabsf(a.w))));
    }
    amax = warp_max(amax);
    const double inv = amax == 0.f ? 0.0 : 127.0 / (double)amax;
    char4* dst = reinterpret_cast<char4*>(q + (size_t)r * k);
    for (int c4 = lane; c4 < n4; c4 += 32) {
      float4 a = src[c4];
      float e[4] = {a.x, a.y, a.z, a.w};
      char4 out;
      int8_t* o = reinterpret_cast<int8_t*>(&out);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        double rr = round((double)e[t] * inv);
        rr = fmin(127.0, fmax(-127.0, rr));
        o[t] = (int8_t)rr;
      }
      dst[c4] = out;
    }
    if (lane == 0) scale[r] = amax == 0.f ? 0.f : __fdiv_rn(amax, 127.0f);
  }
}

// Copies the CLS row (first token) of every sequence into a compact buffer
// (f32 or f16 rows; 16-byte vectors).
template <typename T>
__global__ void gather_rows_kernel(const T* __restrict__ x, const int* __restrict__ cu, int nseq,
                                   int h, T* __restrict__ xc) {
  pdl_wait();
  pdl_trigger();
  const int nv = h * (int)sizeof(T) / 16;
  const size_t total = (size_t)nseq * nv;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int s = (int)(i / nv), c = (int)(i % nv);
    reinterpret_cast<uint4*>(xc + (size_t)s * h)[c] =
        reinterpret_cast<const uint4*>(x + (size_t)cu[s] * h)[c];
  }
}

__device__ __forceinline__ double block_sum_d(double v, double* red) {
  v = warp_sum_d(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

// One CTA per sequence. x holds the final hidden rows: packed [T, h] (mean
// pooling, row cu[s]+t) or compact [nseq, h] (CLS pooling, row s).
// out_dim < h selects matryoshka truncation; mat_ln applies the parameter-
// free LayerNorm (eps 1e-5) first; normalize applies L2 in float64.
__global__ void __launch_bounds__(256)
    pool_kernel(const float* __restrict__ x, const int* __restrict__ cu, int h, int mean_pool,
                int out_dim, int mat_ln, int normalize, float* __restrict__ out) {
  extern __shared__ float pooled[];  // [h]
  __shared__ double red[32];
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x;
  if (mean_pool) {
    const int s0 = cu[s], L = cu[s + 1] - s0;
    const float inv = __fdiv_rn(1.0f, (float)L);
    for (int c = threadIdx.x; c < h; c += blockDim.x) {
      float acc = 0.f;
      for (int t = 0; t < L; ++t) acc = fadd(acc, x[(size_t)(s0 + t) * h + c]);
      pooled[c] = fmul(acc, inv);
    }
  } else {
    for (int c = threadIdx.x; c < h; c += blockDim.x) pooled[c] = x[(size_t)s * h + c];
  }
  __syncthreads();
  int d = h;
  if (out_dim != 0 && out_dim != h) {
    if (mat_ln) {
      double sum = 0.0;
      for (int c = threadIdx.x; c < h; c += blockDim.x) sum += (double)pooled[c];
      const double mean = block_sum_d(sum, red) / (double)h;
      double var = 0.0;
      for (int c = threadIdx.x; c < h; c += blockDim.x) {
        const double dd = (double)pooled[c] - mean;
        var += dd * dd;
      }
      var = block_sum_d(var, red) / (double)h;
      const float inv = (float)(1.0 / sqrt(var + (double)1e-5f));
      const float mf = (float)mean;
      __syncthreads();
      for (int c = threadIdx.x; c < h; c += blockDim.x) pooled[c] = fmul(fsub(pooled[c], mf), inv);
      __syncthreads();
    }
    d = out_dim;
  }
  float scale = 1.0f;
  if (normalize) {
    double ss = 0.0;
    for (int c = threadIdx.x; c < d; c += blockDim.x) ss += (double)pooled[c] * (double)pooled[c];
    ss = block_sum_d(ss, red);
    if (ss > 0) scale = (float)(1.0 / sqrt(ss));
  }
  for (int c = threadIdx.x; c < d; c += blockDim.x)
    out[(size_t)s * d + c] = normalize ? fmul(pooled[c], scale) : pooled[c];
}

// f32 → f16 (round to nearest, saturating at ±65504): GEMM weights of the
// float path.
__global__ void f32_to_f16_kernel(const float* __restrict__ in, size_t n, __half* __restrict__ out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = __float2half_rn(fminf(fmaxf(in[i], -65504.0f), 65504.0f));
}

// f16 → f32 (exact): F16 weights the int8 path quantises as f32 rows.
__global__ void f16_to_f32_kernel(const __half* __restrict__ in, size_t n, float* __restrict__ out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = __half2float(in[i]);
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ in, size_t n,
                                   __nv_bfloat16* __restrict__ out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16_rn(in[i]);
}

}  // namespace futon
