/*
 * futon_oracle.h — CPU restatement of futon's encoder forward pass.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * path in futon_b200/csrc. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py may load it. The product path
 * never calls it and has no CPU fallback.
 *
 * Parity pin: the restatement is checked against the reference's own golden
 * vectors (native/testdata/toy/expected.json, produced by upstream torch
 * code) under the reference's gates (cos >= 0.99999, |d| <= 2e-4,
 * native/model_test.go:19-22). The reference itself is Go and cannot be
 * built in this container (no Go toolchain, no module cache).
 *
 * Reference files restated (paths within github.com/bobbyhiddn/futon):
 *   native/model.go:346-457   EncodeTokensKernel (embed, layers, pool, L2)
 *   native/model.go:550-635   layerForward (post-LN block)
 *   native/model.go:646-739   attendHead, rotateHalf, softmaxScaled
 *   native/model.go:743-769   layerNormRows
 *   native/model.go:306-318   precomputeRoPE
 *   native/kernel.go:223-283  matMulTRows (goKernel summation order)
 *   native/kernel_avx2_amd64.s:20-111  dot4x2f32 panel (CPU baseline only)
 *   native/mathf32.go:40-120  expF32, erfcPos, geluF32, sigmoidF32
 *   native/quant.go:42-137    quantizeRowQ8, quantizeQ8, matMulTQ8
 *   native/config.go:111-116  EffectiveMaxSeqLen
 */
#ifndef FUTON_ORACLE_H
#define FUTON_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Architecture fields of PackConfig (native/config.go:54-102) that the
 * forward reads. */
typedef struct {
    int hidden;         /* hidden_size */
    int num_layers;     /* num_layers */
    int num_heads;      /* num_heads */
    int inter;          /* intermediate_size */
    int vocab;          /* vocab_size */
    int type_vocab;     /* type_vocab_size (0 = no token-type table) */
    int max_seq_len;    /* max_seq_len (rows of the absolute table) */
    int max_trained;    /* max_trained_positions (0 = unset) */
    double eps;         /* layer_norm_eps as declared (converted to f32 like model.go:395) */
    int rope;           /* position_encoding: 1 = "rope", 0 = "absolute" */
    double rope_theta;  /* rope_theta */
    int swiglu;         /* activation: 1 = "swiglu", 0 = "gelu" */
    int pool_mean;      /* pooling: 1 = "mean", 0 = "cls" */
    int normalize;      /* normalize */
    int matryoshka;     /* 1 when the pack declares a matryoshka block */
    int matryoshka_ln;  /* matryoshka.layernorm */
} fo_cfg;

/* Per-layer tensor slots, in the order the flat table passes them. */
enum {
    FO_L_QKV_W = 0, FO_L_QKV_B, FO_L_OUT_W, FO_L_OUT_B, FO_L_NORM1_W, FO_L_NORM1_B,
    FO_L_FC1_W, FO_L_FC1_B, FO_L_GATE_W, FO_L_GATE_B, FO_L_FC2_W, FO_L_FC2_B,
    FO_L_NORM2_W, FO_L_NORM2_B, FO_L_COUNT
};
/* Model-level slots before the per-layer blocks. */
enum { FO_WORD = 0, FO_POS, FO_TYPE, FO_EMB_NORM_W, FO_EMB_NORM_B, FO_GLOBAL_COUNT };

/* GEMM summation order used by the oracle's forward. */
enum {
    FO_GEMM_GO = 0,   /* goKernel matMulTRows order (kernel.go:223-283) — parity */
    FO_GEMM_AVX2 = 1  /* avx2Kernel dot4x2f32 panel order — CPU baseline */
};

typedef struct fo_model fo_model;

/* Builds a model over caller-owned float32 tensors (not copied).
 * tensors has FO_GLOBAL_COUNT + num_layers*FO_L_COUNT entries; absent
 * optional tensors are NULL. q8 != 0 requantises the five layer GEMM
 * weights per row (quant.go:42-86, model.go:265-289), owned by the model.
 * Returns NULL and writes err on failure. */
fo_model *fo_create(const fo_cfg *cfg, const float *const *tensors, int q8,
                    int gemm_mode, char *err, size_t errlen);
void fo_destroy(fo_model *m);

/* Effective max sequence length (config.go:111-116). */
int fo_effective_max_seq_len(const fo_model *m);

/* One sequence forward (model.go:346-457). out receives outDim floats
 * (outDim 0 = hidden). Returns 0 or -1 with err set. */
int fo_encode(const fo_model *m, const int32_t *ids, int n, int out_dim,
              float *out, char *err, size_t errlen);

/* Batch of packed sequences; one independent forward per sequence on a
 * pool of `threads` workers, longest first (provider.go:152-202).
 * out is [nseq, out_dim or hidden]. Returns 0 or -1 (first error). */
int fo_encode_batch(const fo_model *m, const int32_t *ids, const int32_t *cu_seqlens,
                    int nseq, int out_dim, float *out, int threads,
                    char *err, size_t errlen);

/* Read access to the requantised weights (q8 models only): layer li, slot
 * 0..4 = qkv, out, fc1, gate, fc2. Returns NULL when absent. */
const int8_t *fo_q8_data(const fo_model *m, int li, int slot);
const float *fo_q8_scale(const fo_model *m, int li, int slot);

/* Kernel-level restatements, exposed for unit parity tests. */
void fo_matmul_t(float *dst, const float *a, const float *b, int m, int n, int k,
                 const float *bias);
void fo_matmul_t_avx2(float *dst, const float *a, const float *b, int m, int n, int k,
                      const float *bias);
float fo_quantize_row_q8(int8_t *dst, const float *src, int n);
void fo_matmul_t_q8_prequant(float *dst, const int8_t *qa, const float *a_scale,
                             const int8_t *qb, const float *b_scale, int m, int n, int k,
                             const float *bias);
void fo_matmul_t_q8_prequant_scalar(float *dst, const int8_t *qa, const float *a_scale,
                                    const int8_t *qb, const float *b_scale, int m, int n, int k,
                                    const float *bias);
void fo_matmul_t_q8(float *dst, const float *a, const int8_t *qb, const float *scales,
                    int m, int n, int k, const float *bias);
void fo_layernorm_rows(float *x, int rows, int h, const float *w, const float *b, float eps);
void fo_softmax_scaled(float *row, int n, float scale);
float fo_exp(float x);
float fo_gelu(float x);
float fo_sigmoid(float x);
void fo_rope_tables(int max_seq, int head_dim, double theta, float *cos_out, float *sin_out);
/* attendHead (model.go:646-701) for head `head` of one sequence: qkv is its
 * [seq, 3h] float32 block, the first `rows` queries attend over all seq keys,
 * out receives [rows, hd]. rope_cos/rope_sin ([seq or more, hd/2]) are NULL
 * for absolute-position packs. Returns 0, or -1 on a bad shape. */
int fo_attend_head(const float *qkv, int seq, int rows, int h, int hd, int head,
                   const float *rope_cos, const float *rope_sin, int gemm_mode, float *out);
int fo_has_avx2(void);

#ifdef __cplusplus
}
#endif
#endif
