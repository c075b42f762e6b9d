// Host build of the int8 path's exact-order arithmetic, for CPU tests
// against the oracle: the attention (futon_b200/csrc/attn_exact.cuh: the
// same per-row and per-column routines as attn_exact_softmax_kernel and
// attn_exact_pv_kernel, over the same 64-key tiles, in the same order) and
// the activations of futon_b200/csrc/mathf32.cuh.
// Built by tests/test_exact_host.py with nvcc (host code,
// -ffp-contract=off); test infrastructure only.
#include <cmath>
#include <vector>

#define FUTON_EXACT_HOST_ONLY 1
#include "attn_exact.cuh"

using namespace futon;

namespace {

template <int HD>
void attend(const float* qkv, int seq, int rows, int h, int head, float* out) {
  constexpr int kT = 64, kD = HD / 16;
  const int kp = (seq + 7) & ~7;
  const size_t ld = 3 * (size_t)h;
  const float scale = (float)(1.0 / std::sqrt((double)HD));
  std::vector<float> P((size_t)kp * rows), kt((size_t)kT * HD), vt((size_t)kT * HD), pt(kT);
  for (int r = 0; r < rows; ++r) {
    float q[HD];
    for (int d = 0; d < HD; ++d) q[d] = qkv[(size_t)r * ld + head * HD + d];
    float mx = 0.0f;
    for (int k0 = 0; k0 < seq; k0 += kT) {
      const int n = seq - k0 < kT ? seq - k0 : kT;
      for (int j = 0; j < n; ++j)
        for (int d = 0; d < HD; ++d)
          kt[(size_t)j * HD + d] = qkv[(size_t)(k0 + j) * ld + h + head * HD + d];
      exact_scores_tile<HD>(q, kt.data(), n, k0, P.data() + r, (size_t)rows, &mx);
    }
    exact_softmax_row(P.data() + r, (size_t)rows, seq, kp, scale, mx);
  }
  for (int r = 0; r < rows; ++r)
    for (int g = 0; g < 16; ++g) {
      Fma8 acc[kD];
      for (int i = 0; i < kD; ++i) acc[i].zero();
      for (int k0 = 0; k0 < kp; k0 += kT) {
        const int n = kp - k0 < kT ? kp - k0 : kT;
        for (int j = 0; j < n; ++j) {
          pt[j] = P[(size_t)(k0 + j) * rows + r];
          for (int d = 0; d < HD; ++d)
            vt[(size_t)j * HD + d] =
                k0 + j < seq ? qkv[(size_t)(k0 + j) * ld + 2 * h + head * HD + d] : 0.0f;
        }
        exact_pv_tile<HD, kD>(acc, pt.data(), vt.data(), n, g);
      }
      for (int i = 0; i < kD; ++i) out[(size_t)r * HD + g + 16 * i] = acc[i].fold();
    }
}

}  // namespace

// One head of one sequence: qkv [seq, 3h] (q and k already rotated), the
// first `rows` queries attend over all seq keys; out [rows, hd].
extern "C" int fx_attend_head(const float* qkv, int seq, int rows, int h, int hd, int head,
                              float* out) {
  if (seq <= 0 || rows <= 0 || rows > seq || head < 0 || (head + 1) * hd > h) return -1;
  if (hd == 32) attend<32>(qkv, seq, rows, h, head, out);
  else if (hd == 64) attend<64>(qkv, seq, rows, h, head, out);
  else return -1;
  return 0;
}

// exp_f32 on the host (the device restatement of the reference's expF32).
extern "C" float fx_exp_f32(float x) { return exp_f32(x); }

// The int8 path's activations on the host (the device restatements of the
// reference's geluF32 and sigmoidF32, mathf32.go:40-120).
extern "C" float fx_gelu_f32(float x) { return gelu_f32(x); }
extern "C" float fx_sigmoid_f32(float x) { return sigmoid_f32(x); }

// The bf16 path's fast GELU formula (gelu_fast2's evaluation with an exactly
// rounded reciprocal), for the accuracy bound the design states.
extern "C" float fx_gelu_fast_ref(float x) { return gelu_fast_ref(x); }
