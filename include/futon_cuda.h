/*
 * futon_cuda.h — C ABI of libfuton_cuda, the B200 (sm_100a) encoder forward
 * pass behind futon's native Provider.
 *
 * Plain C types only (no CUDA or torch types in any signature), so cgo,
 * ctypes or any FFI can bind it. Every entry point returns 0 on success or a
 * FUTON_E* code, and writes a UTF-8 message into err[errlen] on failure.
 * Device pointers are passed as plain pointers and streams as void*.
 *
 * Reference interfaces replaced (paths within github.com/bobbyhiddn/futon):
 *   native/model.go:112-295   LoadModel / newModel     -> futon_cuda_model_create
 *   native/model.go:346-457   Model.EncodeTokensKernel -> futon_cuda_encode
 *   native/provider.go:152-202 Provider.EmbedBatch     -> futon_cuda_encode_batch
 *   native/kernel.go:26-36    Kernel.MatMulT           -> futon_cuda_matmul_t
 *   native/quant.go:92-96     q8Kernel.MatMulTQ8       -> futon_cuda_matmul_t_q8
 *   native/quant.go:42-70     quantizeRowQ8            -> futon_cuda_quantize_rows_q8
 */
#ifndef FUTON_CUDA_H
#define FUTON_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
#define FUTON_OK 0
#define FUTON_EINVAL 1    /* bad argument, shape, id or configuration */
#define FUTON_ECUDA 2     /* a CUDA runtime or driver call failed */
#define FUTON_ECANCELED 3 /* *cancel became non-zero (context.Canceled) */
#define FUTON_ENOMEM 4    /* device or pinned host allocation failed */
#define FUTON_EDEVICE 5   /* a kernel reported a device-side error (bounded wait expired) */

/* PackConfig enums (native/config.go:14-30). */
#define FUTON_POS_ABSOLUTE 0
#define FUTON_POS_ROPE 1
#define FUTON_ACT_GELU 0
#define FUTON_ACT_SWIGLU 1
#define FUTON_POOL_CLS 0
#define FUTON_POOL_MEAN 1

/* Tensor dtypes a pack may hold (native/safetensors.go:28-33). */
#define FUTON_DTYPE_F32 0
#define FUTON_DTYPE_F16 1

/* Architecture fields of PackConfig (native/config.go:54-102). The host
 * validates the pack (PackConfig.Validate) before calling create. */
typedef struct futon_cfg {
  int32_t hidden_size;
  int32_t num_layers;
  int32_t num_heads;
  int32_t intermediate_size;
  int32_t vocab_size;
  int32_t type_vocab_size;       /* 0 = no token-type table */
  int32_t max_seq_len;
  int32_t max_trained_positions; /* 0 = unset; clamps the effective max length */
  double layer_norm_eps;
  int32_t position_encoding;     /* FUTON_POS_* */
  double rope_theta;
  int32_t activation;            /* FUTON_ACT_* */
  int32_t pooling;               /* FUTON_POOL_* */
  int32_t normalize;             /* L2-normalise the pooled vector */
  int32_t matryoshka;            /* pack declares matryoshka support */
  int32_t matryoshka_layernorm;  /* parameter-free LN before truncation */
} futon_cfg;

/* One named pack tensor in host memory, canonical names as in
 * native/model.go:189-257 ("embeddings.word", "layers.3.attn.qkv.weight", …). */
typedef struct futon_tensor {
  const char* name;
  int32_t dtype;     /* FUTON_DTYPE_* */
  int32_t ndim;
  int64_t shape[4];
  const void* data;  /* row-major, host memory; read during create only */
} futon_tensor;

typedef struct futon_model futon_model;

/* Number of visible CUDA devices (0 when none). */
int futon_cuda_device_count(void);

/* Uploads the pack to every listed device (one weight replica per device).
 * Shapes, names and the tensor set are checked like newModel
 * (model.go:134-263): a missing, misshapen or unexpected tensor is an error.
 * q8 != 0 requantises the five layer GEMM weights to per-row int8 like the
 * FUTON_NATIVE_Q8=1 load (model.go:265-289). Host buffers are not retained. */
int futon_cuda_model_create(const futon_cfg* cfg, const futon_tensor* tensors, int ntensors,
                            const int* devices, int ndev, int q8, futon_model** out, char* err,
                            size_t errlen);

/* Waits for the model's last queued call on every device, then releases
 * every device buffer. Callers must not race it with encode: a host binding
 * refuses new calls and waits for calls in flight first (Provider.Close). */
void futon_cuda_model_destroy(futon_model* model);

/* Encodes nseq packed sequences on the model's device number `device`
 * (an index into the create-time device list). ids holds Σ lengths token ids,
 * cu_seqlens nseq+1 offsets (cu_seqlens[0] = 0). out receives
 * nseq × (out_dim ? out_dim : hidden) floats. All pointers are host memory.
 * Rejects like EncodeTokens (model.go:348-365): an empty sequence, a length
 * above the effective max, an id outside [0, vocab), out_dim outside
 * [0, hidden], truncation without matryoshka support. *cancel (may be NULL)
 * is polled between micro-batches and layers; non-zero → FUTON_ECANCELED.
 * A call of one micro-batch of at most 32,768 tokens replays a CUDA graph of
 * an earlier call with the same launches (captured on the library's own
 * stream the first time); it polls *cancel at entry and before its
 * micro-batch only. */
int futon_cuda_encode(futon_model* model, int device, const int32_t* ids,
                      const int32_t* cu_seqlens, int nseq, int out_dim, float* out,
                      volatile const int* cancel, char* err, size_t errlen);

/* EmbedBatch over all of the model's devices: sequences are split into
 * contiguous, cost-balanced shards (one per device), each encoded by its own
 * host thread and stream; results are index-aligned in out. */
int futon_cuda_encode_batch(futon_model* model, const int32_t* ids, const int32_t* cu_seqlens,
                            int nseq, int out_dim, float* out, volatile const int* cancel,
                            char* err, size_t errlen);

/* Device-resident variant for callers whose ids already live in HBM:
 * d_ids and d_out are device pointers on that device, cu_seqlens is host
 * memory (it plans the micro-batches). Work is queued on `stream`
 * (cudaStream_t, NULL = the library's stream for that device) and the call
 * returns without waiting; futon_cuda_sync reports completion and errors.
 * Calls on one device run on the GPU in the order they were made, whatever
 * their streams (each call's stream first waits for the previous call's
 * end: they share the device's activation workspace).
 * NULL buffers with nseq > 0 are refused (FUTON_EINVAL) before any launch. */
int futon_cuda_encode_device(futon_model* model, int device, const int32_t* d_ids,
                             const int32_t* cu_seqlens, int nseq, int out_dim, float* d_out,
                             void* stream, char* err, size_t errlen);

/* Waits for all work queued on `device` (and `stream`, if non-NULL) and
 * reports any device-side error recorded since the last call. */
int futon_cuda_sync(futon_model* model, int device, void* stream, char* err, size_t errlen);

/* Number of kernels the library launched on `device` since create
 * (counts every launch of this library's own kernels). */
long long futon_cuda_launch_count(futon_model* model, int device);

/* Bytes the model's calls on `device` copied host→device (*h2d: token ids,
 * micro-batch metadata) and device→host (*d2h: vectors, the device error
 * word) since create (no counterpart in the reference: measurement). */
int futon_cuda_io_bytes(futon_model* model, int device, long long* h2d, long long* d2h, char* err,
                        size_t errlen);

/* ---- Per-stage profiler (no counterpart in the reference: measurement) ----
 * When enabled, every launch on `device` is bracketed by CUDA events and
 * attributed to a stage (embed_ln, gemm_qkv, attention, …) together with its
 * algorithmic FLOPs and bytes. futon_cuda_profile resets the counters and
 * turns recording on (enable != 0) or off; futon_cuda_profile_read waits for
 * the device and returns the totals of one stage. */
int futon_cuda_profile(futon_model* model, int device, int enable, char* err, size_t errlen);
int futon_cuda_profile_read(futon_model* model, int device, int stage, double* ms,
                            long long* launches, double* flops, double* bytes, char* err,
                            size_t errlen);
int futon_cuda_profile_stage_count(void);
const char* futon_cuda_profile_stage_name(int stage);

/* ---- Kernel seam (device pointers, CUDA device `cuda_device`) ----
 * Safe to call from several host threads: calls on one device take turns
 * (they share that device's scratch and error word) and each waits for its
 * stream before returning. */

/* dst[m×n] = a[m×k] · b[n×k]ᵀ (+ bias[n]) on the tcgen05 tensor cores with
 * bf16 operands and f32 accumulation. k % 8 == 0. Uses library-managed
 * scratch for the bf16 operand copies. */
int futon_cuda_matmul_t(int cuda_device, float* dst, const float* a, const float* b, int m, int n,
                        int k, const float* bias, void* stream, char* err, size_t errlen);

/* Q8 GEMM (quant.go:99-137): quantises a per row, then exact int8×int8→s32
 * on the tensor cores, then float32(sum)·(sA·sB) + bias. qb is n×k int8,
 * scales has n entries. k % 16 == 0. Bit-exact with the reference scheme. */
int futon_cuda_matmul_t_q8(int cuda_device, float* dst, const float* a, const int8_t* qb,
                           const float* scales, int m, int n, int k, const float* bias,
                           void* stream, char* err, size_t errlen);

/* Per-row symmetric int8 quantisation of src[rows×k] (quantizeRowQ8). */
int futon_cuda_quantize_rows_q8(int cuda_device, int8_t* dst, float* scales, const float* src,
                                int rows, int k, void* stream, char* err, size_t errlen);

/* futon_cuda_matmul_t_q8 for callers that must not allocate device memory
 * (no counterpart in the reference): a serving loop whose HBM another
 * allocator already holds, or a latency-critical path where cudaMalloc or
 * cudaFree (which synchronises the device) is not acceptable. Same inputs,
 * outputs and bit-exact results as futon_cuda_matmul_t_q8, but the quantised
 * activations and scales go to a fixed 4 MiB array in the library's device
 * image (resident on every GPU that loads the library until exit), so
 * align_up(m·k, 256) + 4·m bytes must fit in 4 MiB; larger shapes are
 * rejected with FUTON_EINVAL. The first call on a device resolves that
 * array's device address; make it before any stream capture. That first
 * call (or any earlier library call that launches a kernel on the device)
 * also loads the library's device code there, which is when the array and
 * the code take their device memory (CUDA loads modules lazily by default):
 * make it before another allocator takes the free HBM. After it, calls
 * allocate nothing; each zeroes its device error word and waits for its
 * stream.
 * All calls on a device share the one array: calls whose GPU work overlaps
 * (other host threads, other streams) race and must be serialised by the
 * caller. */
int futon_cuda_matmul_t_q8_noalloc(int cuda_device, float* dst, const float* a, const int8_t* qb,
                                   const float* scales, int m, int n, int k, const float* bias,
                                   void* stream, char* err, size_t errlen);

/* Cancellation test hook, the library-side form of the reference's
 * cancelAfterN test context (native/model_test.go:203-244): the next
 * futon_cuda_encode / futon_cuda_encode_device call made from this host
 * thread passes `polls` cancellation checkpoints (the entry check, then one
 * per micro-batch, one before each layer and one before each layer's FFN)
 * and reports FUTON_ECANCELED at the next, as if *cancel had been raised
 * there. The countdown then disarms; polls < 0 disarms it at once. */
void futon_cuda_debug_cancel_after(long long polls);

/* Failure-detection self-test (no counterpart in the reference): launches
 * one CTA that waits, through the same bounded-wait routine every pipeline
 * kernel uses, on an mbarrier phase that nothing completes. The wait gives up
 * after its 1 s limit, records its code in the device error word and the
 * kernel returns, so the call returns FUTON_EDEVICE ("device wait timed out")
 * with the context still usable. Any other outcome is an error of the
 * library's failure detection on this device (FUTON_ECUDA). */
int futon_cuda_selftest_wait_timeout(int cuda_device, char* err, size_t errlen);

#ifdef __cplusplus
}
#endif
#endif /* FUTON_CUDA_H */
