// mathf32.cuh — device versions of futon's float32 transcendentals.
//
// Restates native/mathf32.go:40-124 (futon, MIT): expF32 is Cephes' single-
// precision exp (range reduction k·ln2 + r, minimax polynomial, scale by
// 2^k); erfcPos is the Numerical Recipes erfcc Chebyshev fit; geluF32 is the
// exact-erf GELU evaluated through erfc; sigmoidF32 is 1/(1+e^-x) with the
// reference's clamps. Every multiply and add is a separately rounded f32 op
// (__fmul_rn / __fadd_rn), the evaluation the Go source has on amd64, so the
// device activations equal the CPU oracle's bit for bit.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <cstdint>
#include <cstring>

// FUTON_HD marks the exact-order f32 primitives that host code can call too
// (CPU unit tests of the device arithmetic compile them with a host C++
// compiler and -ffp-contract=off); device code is unchanged by it.
#if defined(__CUDACC__)
#define FUTON_HD __host__ __device__
#else
#define FUTON_HD
#endif

namespace futon {

FUTON_HD __forceinline__ float fmul(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}
FUTON_HD __forceinline__ float fadd(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fadd_rn(a, b);
#else
  return a + b;
#endif
}
FUTON_HD __forceinline__ float fsub(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fsub_rn(a, b);
#else
  return a - b;
#endif
}
FUTON_HD __forceinline__ float fdiv(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fdiv_rn(a, b);
#else
  return a / b;
#endif
}
FUTON_HD __forceinline__ float f32_from_bits(int32_t b) {
#ifdef __CUDA_ARCH__
  return __int_as_float(b);
#else
  float f;
  std::memcpy(&f, &b, sizeof f);
  return f;
#endif
}

constexpr float kExpOverflowF32 = 88.72283f;   // ln(MaxFloat32)
constexpr float kExpUnderflowF32 = -87.33654f; // ln(2^-126)
constexpr float kExpClampLo = -104.0f;

FUTON_HD __forceinline__ float exp_f32(float x) {
  if (x < kExpUnderflowF32) return 0.0f;
  float kf = fsub(fadd(fmul(x, 1.4426950408889634f), 12582912.0f), 12582912.0f);
  int32_t k = (int32_t)kf;
  float r = fsub(x, fmul(kf, 0.693145751953125f));
  r = fsub(r, fmul(kf, 1.428606820309417e-06f));
  float p = 1.9875691500e-4f;
  p = fadd(fmul(p, r), 1.3981999507e-3f);
  p = fadd(fmul(p, r), 8.3334519073e-3f);
  p = fadd(fmul(p, r), 4.1665795894e-2f);
  p = fadd(fmul(p, r), 1.6666665459e-1f);
  p = fadd(fmul(p, r), 5.0000001201e-1f);
  p = fadd(fmul(fadd(fmul(p, r), 1.0f), r), 1.0f);
  int32_t e = k + 127;
  if (e <= 0) return 0.0f;
  if (e >= 255) return fmul(fmul(p, f32_from_bits((e - 1) << 23)), 2.0f);
  return fmul(p, f32_from_bits(e << 23));
}

FUTON_HD __forceinline__ float erfc_pos_f32(float a) {
  float t = fdiv(1.0f, fadd(1.0f, fmul(0.5f, a)));
  float p = 0.17087277f;
  p = fsub(fmul(p, t), 0.82215223f);
  p = fadd(fmul(p, t), 1.48851587f);
  p = fsub(fmul(p, t), 1.13520398f);
  p = fadd(fmul(p, t), 0.27886807f);
  p = fsub(fmul(p, t), 0.18628806f);
  p = fadd(fmul(p, t), 0.09678418f);
  p = fadd(fmul(p, t), 0.37409196f);
  p = fadd(fmul(p, t), 1.00002368f);
  p = fsub(fmul(p, t), 1.26551223f);
  float e = fsub(p, fmul(a, a));
  if (e < kExpClampLo) e = kExpClampLo;
  return fmul(t, exp_f32(e));
}

FUTON_HD __forceinline__ float gelu_f32(float x) {
  float a = fmul(x, 0.7071067811865476f);
  if (a < 0) a = -a;
  float c = erfc_pos_f32(a);
  if (x < 0) return fmul(fmul(0.5f, x), c);
  return fmul(fmul(0.5f, x), fsub(2.0f, c));
}

FUTON_HD __forceinline__ float sigmoid_f32(float x) {
  float e = -x;
  if (e < kExpClampLo) e = kExpClampLo;
  if (e > kExpOverflowF32) return 0.0f;
  return fdiv(1.0f, fadd(1.0f, exp_f32(e)));
}

// Fast variants for the float path, whose outputs are rounded to f16 (2^-11
// relative) right after. GELU: erfc(z) = 1 / P(z)^16 with the degree-6
// polynomial of Abramowitz & Stegun 7.1.28 (|error| ≤ 3e-7; ≤ 7.1e-7 on
// gelu over [−12, 12] in f32), one hardware reciprocal and no exponential;
// P^16 overflowing to +inf gives erfc = 0, the correct limit.
// SiLU: g · 1/(1 + 2^(−g·log2 e)).
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Paired f32 arithmetic (sm_100 f32x2: one instruction, two lanes).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// GELU of two values. With z = |x| and the 7.1.28 coefficients a_k scaled
// by (1/√2)^k · 2^(1/16), P'(z)^16 = 2 · P(z/√2)^16, so q = 1/P'(z)^16 =
// 0.5 · erfc(|x|/√2) and gelu(x) = max(x, 0) − |x| · q for either sign.
// gelu_p(k): P' coefficient k, from z^6 (k = 0) down to z^0 (k = 6).
FUTON_HD constexpr float gelu_p(int k) {
  return k == 0   ? 5.6212996640e-06f
         : k == 1 ? 5.1055209009e-05f
         : k == 2 ? 3.9686137011e-05f
         : k == 3 ? 3.4227392389e-03f
         : k == 4 ? 2.2076998457e-02f
         : k == 5 ? 5.2075163037e-02f
                  : 1.0442737824e+00f;
}

// The same evaluation on one value with an exactly rounded reciprocal
// (gelu_fast2 uses rcp.approx, within 1 ulp of it): the host's check of the
// formula's accuracy.
FUTON_HD __forceinline__ float gelu_fast_ref(float x) {
  const float z = x < 0.0f ? -x : x;
  float p = gelu_p(0);
  for (int k = 1; k < 7; ++k) p = fmaf(p, z, gelu_p(k));
  p = p * p;
  p = p * p;
  p = p * p;
  p = p * p;
  return fmaf(-z, 1.0f / p, x > 0.0f ? x : 0.0f);
}

__device__ __forceinline__ void gelu_fast2(float& x0, float& x1) {
  const float z0 = fabsf(x0), z1 = fabsf(x1);
  const uint64_t z = f2_pack(z0, z1);
  uint64_t p = f2_fma(f2_pack(gelu_p(0), gelu_p(0)), z, f2_pack(gelu_p(1), gelu_p(1)));
  p = f2_fma(p, z, f2_pack(gelu_p(2), gelu_p(2)));
  p = f2_fma(p, z, f2_pack(gelu_p(3), gelu_p(3)));
  p = f2_fma(p, z, f2_pack(gelu_p(4), gelu_p(4)));
  p = f2_fma(p, z, f2_pack(gelu_p(5), gelu_p(5)));
  p = f2_fma(p, z, f2_pack(gelu_p(6), gelu_p(6)));
  p = f2_mul(p, p);
  p = f2_mul(p, p);
  p = f2_mul(p, p);
  p = f2_mul(p, p);
  float p0, p1;
  f2_unpack(p, p0, p1);
  x0 = fmaf(-z0, rcp_approx(p0), fmaxf(x0, 0.0f));
  x1 = fmaf(-z1, rcp_approx(p1), fmaxf(x1, 0.0f));
}

__device__ __forceinline__ float gelu_fast(float x) {
  float y = 0.0f;
  gelu_fast2(x, y);
  return x;
}

__device__ __forceinline__ float silu_fast(float g) {
  const float e = exp2_approx(fminf(-g, 80.0f) * 1.4426950408889634f);
  return g * rcp_approx(1.0f + e);
}

}  // namespace futon
