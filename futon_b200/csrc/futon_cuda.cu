// futon_cuda.cu — libfuton_cuda: model upload, forward orchestration and the
// C ABI declared in include/futon_cuda.h.
//
// Data layout in HBM, per device (one full replica per GPU):
//   embeddings: word [vocab, h] f32, position [max_seq, h] f32 (absolute
//     packs), token-type row 0 [h] f32, embedding LayerNorm γ/β f32;
//   per layer: qkv W [3h, h], out W [h, h], fc1 W [inter, h] (or fc1‖gate
//     interleaved [2·inter, h] for SwiGLU), fc2 W [h, inter] — f16, K-major
//     (the pack's nn.Linear layout), or int8 + per-row f32 scales on the Q8
//     path; biases and LayerNorm parameters f32;
//   rotary cos/sin tables [max_trained, hd/2] f32 (RoPE packs).
// Activations of one micro-batch of T packed tokens: the residual stream —
// xb [T, h] f16 on the float path (also the GEMMs' A operand, updated in
// place by the fused residual + LayerNorm epilogues), x [T, h] f32 plus its
// int8 codes on the Q8 path — qkv [T, 3h], attn [T, h], ffn [T, inter],
// xf [T, h] f32 (final hidden rows for pooling), tmp [T, h] f32
// (pre-LayerNorm sums where LayerNorm is not fused).
//
// One forward = embed+LN, then per layer: qkv GEMM, attention, out GEMM with
// residual, LN, fc1 GEMM with GELU or SwiGLU, fc2 GEMM with residual, LN;
// then one pooling kernel. The last layer of a CLS-pooled pack runs its
// query-side work on the CLS rows only (native/model.go:403-410).
#include "../../include/futon_cuda.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <functional>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "attention.cuh"
#include "attention_tc2.cuh"
#include "attn_exact.cuh"
#include "common.cuh"
#include "gemm_launch.cuh"
#include "rowops.cuh"

using namespace futon;
using bf16 = __nv_bfloat16;  // the MatMulT seam's operands
using f16 = __half;          // the float path's operands and activations

// Element type of a 2-D TMA operand.
enum Elem : uint32_t { kElemS8 = 1, kElemBf16 = 2, kElemF16 = 3 };

namespace {

int set_err(char* err, size_t errlen, int code, const char* fmt, ...) {
  if (err && errlen) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, errlen, fmt, ap);
    va_end(ap);
  }
  return code;
}

// The tail of every C entry point: no C++ exception crosses the ABI (a cgo
// or ctypes caller cannot take one); host allocation failure is
// FUTON_ENOMEM, anything else FUTON_ECUDA with its message.
#define FUTON_CATCH(err, errlen)                                                         \
  catch (const std::bad_alloc&) {                                                        \
    return set_err(err, errlen, FUTON_ENOMEM, "native: out of host memory");             \
  }                                                                                      \
  catch (const std::exception& ex_) {                                                    \
    return set_err(err, errlen, FUTON_ECUDA, "native: host exception: %s", ex_.what());  \
  }                                                                                      \
  catch (...) {                                                                          \
    return set_err(err, errlen, FUTON_ECUDA, "native: host exception");                  \
  }

#define CU_TRY(call)                                                                     \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return set_err(err, errlen, e_ == cudaErrorMemoryAllocation ? FUTON_ENOMEM : FUTON_ECUDA, \
                     "native: cuda %s (%s:%d)", cudaGetErrorString(e_), __FILE__, __LINE__); \
  } while (0)

// ---------------------------------------------------------------------------
// Tensor maps (TMA descriptors)
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D row-major [rows, cols] operand (int8, bf16 or f16) read in
// 128-byte-wide, box_rows-high swizzled tiles. Rows and columns past the
// extent read as 0.
bool make_operand_map(CUtensorMap* map, const void* base, Elem e, uint64_t rows, uint64_t cols,
                      uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const bool s8 = e == kElemS8;
  const uint32_t esz = s8 ? 1 : 2;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * esz};
  cuuint32_t box[2] = {128u / esz, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = s8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : e == kElemF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// f16 [rows, cols] GEMM output (row stride ld) written by TMA tile stores:
// 32 × 32 boxes with the 64-byte swizzle the epilogue staging uses.
bool make_output_map(CUtensorMap* map, void* base, uint64_t rows, uint64_t cols, uint64_t ld) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The attention kernels' view of the [T, 3h] f16 qkv buffer:
// box_rows × hd tiles with the swizzle spanning one tile row (64 B for hd 32,
// 128 B for hd 64). Rows past T read as 0.
bool make_qkv_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, int hd,
                  uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)hd, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  hd == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Column-slice width of the fused LayerNorm GEMMs (128-column slices, which
// leave room for a fourth pipeline stage, measured 25 % slower on the bge
// shape: three-CTA clusters and a third copy of every A tile).
int ln_slice_cols(int) { return 192; }

// N tile for a GEMM with N output columns: the widest of 256/192/128 that
// divides N, else 64 (partial last tile, masked in the epilogue).
int pick_bn(int n) {
  if (n % 256 == 0) return 256;
  if (n % 192 == 0) return 192;
  if (n % 128 == 0) return 128;
  return 64;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Tensor maps of activation buffers, memoised per device: a map is a pure
// function of its encode arguments (kind, base address, extents, box), so a
// hit returns exactly what encoding again would. Calls with the same batch
// shape (a serving loop, benchmark repeats) then encode nothing on the host.
struct MapKey {
  int kind;
  const void* base;
  uint64_t a, b, c, d;
  bool operator==(const MapKey& o) const {
    return kind == o.kind && base == o.base && a == o.a && b == o.b && c == o.c && d == o.d;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = 1469598103934665603ull;
    auto mix = [&](uint64_t v) { h = (h ^ v) * 1099511628211ull; };
    mix((uint64_t)k.kind);
    mix((uint64_t)(uintptr_t)k.base);
    mix(k.a);
    mix(k.b);
    mix(k.c);
    mix(k.d);
    return (size_t)h;
  }
};
struct MapCache {
  std::unordered_map<MapKey, CUtensorMap, MapKeyHash> maps;
  template <typename Make>
  bool get(const MapKey& k, CUtensorMap* out, Make&& make) {
    auto it = maps.find(k);
    if (it != maps.end()) {
      *out = it->second;
      return true;
    }
    if (!make(out)) return false;
    if (maps.size() >= 4096) maps.clear();  // many distinct batch shapes: start over
    maps.emplace(k, *out);
    return true;
  }
};
enum MapKind : int { kMapOperand = 1, kMapOutput = 2, kMapQkv = 3 };

// ---------------------------------------------------------------------------
// Model state
// ---------------------------------------------------------------------------
struct GemmWeight {
  void* w = nullptr;        // f16 [n, k] or int8 [n, k]
  float* scale = nullptr;   // int8 only: [n]
  float* bias = nullptr;    // [n] or null
  int n = 0, k = 0, bn = 64;
  // pair: the f16 forward runs this weight's GEMMs as CTA-pair tiles
  // (gemm_tc_kernel<..., PAIR>), whose CTAs each stage bn / 2 rows: the
  // map's box is bn / 2 rows then, else bn (bn / 2 above 256).
  bool pair = false;
  CUtensorMap map;
};

struct LayerDev {
  GemmWeight qkv, out, fc1, fc2;  // fc1 is fc1‖gate interleaved for SwiGLU
  float *n1w, *n1b, *n2w, *n2b;
};

// Float path: the residual stream is xb (f16), updated in place by the
// fused residual + LayerNorm epilogues; xf receives the f32 final hidden
// state for pooling. Int8 path: the residual stream is x (f32) plus its int8
// codes xq/xs; xb is unused.
struct Workspace {
  size_t tokens = 0;  // capacity
  void* base = nullptr;
  float* x;          // int8 path: residual stream (f32)
  f16* xb;           // float path: residual stream / GEMM operand (f16)
  float* xf;         // float path: final hidden rows (f32) for pooling
  void* qkv;         // f16 (float path) or f32 (q8 path)
  void* attn;        // f16 (float path) or f32 (q8 path)
  void* ffn;         // f16 or f32
  float* tmp;        // pre-LayerNorm sums when LayerNorm is not fused
  void* xc;          // CLS rows of the residual stream (f16 or f32)
  int8_t *xq, *attnq, *ffnq;
  float *xs, *attns, *ffns;
};

struct DevCtx {
  int device = 0;
  // Set while a small float-path call's forward is captured into a graph:
  // its launches carry programmatic stream serialization (launch_k).
  bool pdl = false;
  std::vector<int> plan_slots;  // upload_mb_meta's counting-sort slots
  int num_sms = 148;
  bool gemm_pair = false;  // the model's gemm_pair option, read by upload_gemm
  cudaStream_t stream = nullptr;
  std::mutex mu;
  std::vector<void*> allocs;
  float *word = nullptr, *pos = nullptr, *type0 = nullptr, *embw = nullptr, *embb = nullptr;
  float *rcos = nullptr, *rsin = nullptr;
  std::vector<LayerDev> layers;
  int* err_word = nullptr;
  Workspace ws;
  // call-scoped buffers
  int* d_ids = nullptr;
  size_t d_ids_cap = 0;
  int* d_meta = nullptr;
  size_t d_meta_cap = 0;
  float* d_out = nullptr;
  size_t d_out_cap = 0;
  float* d_pscr = nullptr;  // exact int8-path attention: rows of P for a head group
  size_t d_pscr_cap = 0;
  int* h_meta = nullptr;  // pinned
  size_t h_meta_cap = 0;
  int* h_ids = nullptr;   // pinned
  size_t h_ids_cap = 0;
  float* h_out = nullptr; // pinned
  size_t h_out_cap = 0;
  int* h_err = nullptr;   // pinned: the device error word, read back after a call
  size_t h_err_cap = 0;
  cudaEvent_t meta_evt = nullptr;
  // Recorded on a call's stream after its last launch; the next call's stream
  // waits on it first. Calls may use different streams (encode_device takes
  // the caller's), and they share the workspace and the meta buffer.
  cudaEvent_t done_evt = nullptr;
  MapCache map_cache;  // activation tensor maps (guarded by mu)
  std::vector<cudaEvent_t> out_evts;  // host-buffer calls: one per micro-batch's D2H
  std::atomic<long long> launches{0};
  // Bytes this device's calls copied host→device and device→host (ids,
  // micro-batch metadata, vectors, the device error word).
  std::atomic<long long> h2d_bytes{0}, d2h_bytes{0};
  // Optional per-stage profiler (CUDA events around each launch).
  bool prof_on = false;
  struct ProfRec { cudaEvent_t a, b; int stage; double flops, bytes; };
  std::vector<ProfRec> prof_pending;
  std::vector<cudaEvent_t> ev_pool, ev_all;
  struct ProfAgg { double ms = 0, flops = 0, bytes = 0; long long n = 0; };
  ProfAgg prof_agg[16];
  // CUDA graphs of small host-buffer calls: the launches of a one-micro-batch
  // forward, keyed by every value they were captured with (shapes, metadata
  // offsets, buffer addresses, stream), replayed when a call repeats them.
  struct GraphEntry {
    cudaGraphExec_t exec = nullptr;
    long long launches = 0;  // kernels in the graph
    unsigned long long used = 0;
  };
  std::map<std::vector<long long>, GraphEntry> graphs;
  unsigned long long graph_clock = 0;

  ~DevCtx() {
    cudaSetDevice(device);
    if (done_evt) cudaEventSynchronize(done_evt);  // the last call, whatever its stream
    if (stream) cudaStreamSynchronize(stream);
    for (auto& kv : graphs) cudaGraphExecDestroy(kv.second.exec);
    for (cudaEvent_t e : out_evts) cudaEventDestroy(e);
    for (void* p : allocs) cudaFree(p);
    if (ws.base) cudaFree(ws.base);
    if (d_ids) cudaFree(d_ids);
    if (d_meta) cudaFree(d_meta);
    if (d_out) cudaFree(d_out);
    if (d_pscr) cudaFree(d_pscr);
    if (h_meta) cudaFreeHost(h_meta);
    if (h_ids) cudaFreeHost(h_ids);
    if (h_out) cudaFreeHost(h_out);
    if (h_err) cudaFreeHost(h_err);
    if (meta_evt) cudaEventDestroy(meta_evt);
    if (done_evt) cudaEventDestroy(done_evt);
    for (cudaEvent_t e : ev_all) cudaEventDestroy(e);
    if (stream) cudaStreamDestroy(stream);
  }
};

}  // namespace

struct futon_model {
  futon_cfg cfg;
  int q8 = 0;
  // Residual + LayerNorm fused into the out/fc2 GEMMs: hidden = w·P with
  // slice width w = ln_slice_cols(hidden) and 2 ≤ P ≤ 4 (P CTAs of a
  // cluster share each row tile).
  bool fuse_ln = false;
  int head_dim = 0;
  int eff_max = 0;
  int swiglu_half = 0;
  // Attention kernel of the float path (read from FUTON_CUDA_ATTN when the
  // model is created): 0 = attn_heads_kernel, 2 = attn_tc2_kernel
  // (head_dim 32 or 64, even head count; others keep 0).
  int attn_kind = 0;
  // FUTON_CUDA_ATTN_SPLIT=1: attn_heads_kernel launches with the head groups
  // shared among grid.y CTAs when the tiles alone would leave SMs idle.
  bool attn_split = true;
  // FUTON_CUDA_Q8_ATTN=exact: the int8 path's attention runs in the
  // reference's exact float32 operation order (attn_exact.cuh).
  bool q8_exact_attn = true;
  // FUTON_CUDA_GEMM_PAIR=1: the float path's GEMMs run as CTA-pair tiles
  // (M = 256 over two SMs, each staging half of every weight tile).
  bool gemm_pair = false;
  std::vector<std::unique_ptr<DevCtx>> devs;
};

namespace {

// Tokens per micro-batch. Measured on the c4 workload (one B200): 131,072 →
// 524,288 tokens is 3.8 % more embeddings/s (a quarter of the launches, each
// with its prologue, pipeline fill and drain, and a quarter of the tails);
// the activations then take ≈ 4.4 GB of workspace for bge-small.
constexpr int kTokenBudget = 524288;
// The exact int8 attention's probability scratch per micro-batch (floats):
// a micro-batch also closes before its Σ pad8(L)·L would pass this, so
// long-sequence batches stay within int offsets and 4 GiB of scratch.
constexpr size_t kExactPBudget = (size_t)1 << 30;

// Cancellation checkpoint: entry, every micro-batch, every layer and every
// layer's FFN (the points where native/model.go checks ctx.Err()). The
// countdown, armed per host thread by futon_cuda_debug_cancel_after, makes
// the checkpoint that follows `n` passed ones report cancellation, as the
// reference's tests do with a context canceled after N Err() checks.
thread_local long long t_cancel_after = -1;

bool canceled(volatile const int* cancel) {
  if (t_cancel_after == 0) {
    t_cancel_after = -1;
    return true;
  }
  if (t_cancel_after > 0) --t_cancel_after;
  return cancel && *cancel;
}

// Profiler stages (futon_cuda_profile_read's `stage` argument).
enum Stage : int {
  kStEmbed = 0, kStGemmQkv, kStAttn, kStAttnCls, kStGather, kStQuant, kStGemmOut, kStLayerNorm,
  kStGemmFc1, kStGemmFc2, kStPool, kNumStages
};
const char* kStageNames[kNumStages] = {"embed_ln", "gemm_qkv", "attention", "attention_cls",
                                       "gather_cls", "quant_rows", "gemm_out", "layernorm",
                                       "gemm_fc1", "gemm_fc2", "pool"};

cudaEvent_t prof_event(DevCtx& d) {
  if (!d.ev_pool.empty()) {
    cudaEvent_t e = d.ev_pool.back();
    d.ev_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  d.ev_all.push_back(e);
  return e;
}
// Brackets one launch when profiling is on.
struct ProfScope {
  DevCtx& d;
  cudaStream_t st;
  int stage;
  double flops, bytes;
  cudaEvent_t a = nullptr;
  ProfScope(DevCtx& d_, cudaStream_t st_, int stage_, double flops_, double bytes_)
      : d(d_), st(st_), stage(stage_), flops(flops_), bytes(bytes_) {
    if (d.prof_on) {
      a = prof_event(d);
      cudaEventRecord(a, st);
    }
  }
  ~ProfScope() {
    if (d.prof_on && a) {
      cudaEvent_t b = prof_event(d);
      cudaEventRecord(b, st);
      d.prof_pending.push_back({a, b, stage, flops, bytes});
    }
  }
};

void prof_collect(DevCtx& d) {
  for (auto& r : d.prof_pending) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
      auto& g = d.prof_agg[r.stage];
      g.ms += ms;
      g.flops += r.flops;
      g.bytes += r.bytes;
      g.n += 1;
    }
    d.ev_pool.push_back(r.a);
    d.ev_pool.push_back(r.b);
  }
  d.prof_pending.clear();
}

int effective_max(const futon_cfg& c) {
  if (c.max_trained_positions > 0 && c.max_trained_positions < c.max_seq_len)
    return c.max_trained_positions;
  return c.max_seq_len;
}

// ---- tensor lookup -------------------------------------------------------
struct HostTensor {
  const futon_tensor* t = nullptr;
  std::vector<float> f32;  // f32 copy of an F16 tensor, made when first asked for as f32
  const float* data();
};

// A GEMM weight as the caller holds it: F32 or F16 (uploaded without an
// f32 copy on the host).
struct HostMat {
  const void* p = nullptr;
  int dtype = FUTON_DTYPE_F32;
};

float f16_to_f32(uint16_t h) {
  // Exact binary16 → binary32 conversion.
  uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      int e = -1;
      do { man <<= 1; ++e; } while (!(man & 0x400));
      bits = sign | (uint32_t)(127 - 15 - e) << 23 | (man & 0x3ff) << 13;
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | man << 13;
  } else {
    bits = sign | (exp + 127 - 15) << 23 | man << 13;
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

// Runs fn(0), …, fn(n-1), each on a host thread of its own where one can be
// started and on the calling thread otherwise, and returns when all have
// finished. No exception escapes: a thread that cannot be started only
// serialises its item.
template <typename Fn>
void run_on_threads(int n, Fn&& fn) {
  std::vector<std::thread> th;
  int started = 0;
  try {
    th.reserve(n);
    for (; started < n; ++started) th.emplace_back(fn, started);
  } catch (...) {
  }
  for (int i = started; i < n; ++i) fn(i);
  for (auto& t : th) t.join();
}

// Expands n binary16 values to binary32 (exact): through a 65,536-entry
// table of f16_to_f32, on up to 16 host threads for large tensors (a real
// pack's weights are F16, so this is most of a cold start's host work).
void f16_expand(const uint16_t* src, size_t n, float* dst) {
  static std::vector<float> table;
  static std::once_flag once;
  std::call_once(once, [] {
    table.resize(65536);
    for (uint32_t h = 0; h < 65536; ++h) table[h] = f16_to_f32((uint16_t)h);
  });
  const float* tb = table.data();
  auto run = [&](size_t lo, size_t hi) {
    for (size_t k = lo; k < hi; ++k) dst[k] = tb[src[k]];
  };
  constexpr size_t kPerThread = size_t(1) << 22;
  const size_t hw = std::max<size_t>(1, std::thread::hardware_concurrency());
  const size_t nt = std::min<size_t>({hw, size_t(16), (n + kPerThread - 1) / kPerThread});
  if (nt <= 1) {
    run(0, n);
    return;
  }
  std::vector<std::thread> th;
  const size_t per = (n + nt - 1) / nt;
  size_t launched = 0;  // chunks [0, launched) run on threads, the rest here
  try {
    for (; launched < nt; ++launched) {
      const size_t lo = launched * per, hi = std::min(n, lo + per);
      if (lo < hi) th.emplace_back(run, lo, hi);
    }
  } catch (...) {  // no thread available: finish on this one
  }
  for (size_t i = launched; i < nt; ++i) run(std::min(n, i * per), std::min(n, i * per + per));
  for (auto& x : th) x.join();
}

const float* HostTensor::data() {
  if (t->dtype == FUTON_DTYPE_F32) return (const float*)t->data;
  if (f32.empty()) {
    size_t n = 1;
    for (int k = 0; k < t->ndim; ++k) n *= (size_t)t->shape[k];
    f32.resize(n);
    f16_expand((const uint16_t*)t->data, n, f32.data());
  }
  return f32.data();
}

struct TensorSet {
  std::map<std::string, HostTensor> byname;
  std::map<std::string, bool> used;
};

// Looks up `name` with shape `shape`; on success *ht is its entry (null if
// optional and absent).
int find_tensor(TensorSet& ts, const std::string& name, const std::vector<int64_t>& shape,
                bool optional, HostTensor** ht, char* err, size_t errlen) {
  *ht = nullptr;
  auto it = ts.byname.find(name);
  if (it == ts.byname.end()) {
    if (optional) return FUTON_OK;
    return set_err(err, errlen, FUTON_EINVAL, "native: missing tensor %s", name.c_str());
  }
  const futon_tensor* t = it->second.t;
  if (t->ndim != (int)shape.size())
    return set_err(err, errlen, FUTON_EINVAL, "native: tensor %s rank %d, want %d", name.c_str(),
                   t->ndim, (int)shape.size());
  for (size_t i = 0; i < shape.size(); ++i)
    if (t->shape[i] != shape[i])
      return set_err(err, errlen, FUTON_EINVAL, "native: tensor %s dim %zu is %lld, want %lld",
                     name.c_str(), i, (long long)t->shape[i], (long long)shape[i]);
  ts.used[name] = true;
  *ht = &it->second;
  return FUTON_OK;
}

int need(TensorSet& ts, const std::string& name, std::vector<int64_t> shape, bool optional,
         const float** out, char* err, size_t errlen) {
  HostTensor* ht;
  int rc = find_tensor(ts, name, shape, optional, &ht, err, errlen);
  *out = ht ? ht->data() : nullptr;
  return rc;
}

// A GEMM weight in the caller's dtype (no f32 copy of F16 data).
int need_mat(TensorSet& ts, const std::string& name, std::vector<int64_t> shape, HostMat* out,
             char* err, size_t errlen) {
  HostTensor* ht;
  int rc = find_tensor(ts, name, shape, false, &ht, err, errlen);
  if (rc) return rc;
  out->p = ht->t->data;
  out->dtype = ht->t->dtype;
  return FUTON_OK;
}

// ---- device uploads ------------------------------------------------------
template <typename T>
int dev_alloc(DevCtx& d, T** p, size_t count, char* err, size_t errlen) {
  void* v = nullptr;
  CU_TRY(cudaMalloc(&v, std::max<size_t>(count * sizeof(T), 16)));
  d.allocs.push_back(v);
  *p = static_cast<T*>(v);
  return FUTON_OK;
}

// Uploads go through d.stream, in order with the kernels that convert them
// (a plain cudaMemcpy from pageable memory may return before its DMA has
// landed, and d.stream does not wait for the legacy stream). The caller
// synchronises d.stream before the source memory goes away.
int upload_f32(DevCtx& d, float** dst, const float* src, size_t count, char* err, size_t errlen) {
  if (!src) { *dst = nullptr; return FUTON_OK; }
  int rc = dev_alloc(d, dst, count, err, errlen);
  if (rc) return rc;
  CU_TRY(cudaMemcpyAsync(*dst, src, count * sizeof(float), cudaMemcpyHostToDevice, d.stream));
  return FUTON_OK;
}

// Uploads a GEMM weight (optionally two interleaved halves for SwiGLU) as
// f16 or int8 + per-row scales, builds its bias and its TMA descriptor.
// F16 weights of the float path go to the device as they are (exact: no
// rounding and no host f32 copy); F32 weights are rounded to f16 on the
// device; the int8 path quantises f32 rows (F16 weights are widened on the
// device first). staging: device scratch of ≥ 6 bytes per weight element.
// ln_slices: the GEMM feeds the fused LayerNorm epilogue, which splits each
// row into 192-column slices held by the CTAs of one cluster.
int upload_gemm(DevCtx& d, GemmWeight& g, HostMat w1, const float* b1, HostMat w2,
                const float* b2, int n1, int k, int half, bool q8, bool ln_slices, void* staging,
                char* err, size_t errlen) {
  const bool two = w2.p != nullptr;
  const int n = two ? 2 * n1 : n1;
  g.n = n;
  g.k = k;
  if (two && w2.dtype != w1.dtype)
    return set_err(err, errlen, FUTON_EINVAL, "native: fc1 and gate weights differ in dtype");
  const bool in16 = w1.dtype == FUTON_DTYPE_F16;
  const size_t esz = in16 ? 2 : 4, count = (size_t)n * k;
  float* st32 = static_cast<float*>(staging);
  uint8_t* st16 = static_cast<uint8_t*>(staging) + count * 4;
  int rc;
  f16* w16 = nullptr;
  if (!q8 && (rc = dev_alloc(d, &w16, count, err, errlen))) return rc;
  // The matrix as given (interleaving fc1/gate blocks of `half` rows): F16
  // straight into the float path's weight, else into staging.
  uint8_t* dst = (!q8 && in16) ? reinterpret_cast<uint8_t*>(w16)
                               : (in16 ? st16 : reinterpret_cast<uint8_t*>(st32));
  if (!two) {
    CU_TRY(cudaMemcpyAsync(dst, w1.p, count * esz, cudaMemcpyHostToDevice, d.stream));
  } else {
    const size_t blk = (size_t)half * k * esz;
    for (int j = 0; j * half < n1; ++j) {
      CU_TRY(cudaMemcpyAsync(dst + (size_t)(2 * j) * blk, (const uint8_t*)w1.p + (size_t)j * blk,
                             blk, cudaMemcpyHostToDevice, d.stream));
      CU_TRY(cudaMemcpyAsync(dst + (size_t)(2 * j + 1) * blk,
                             (const uint8_t*)w2.p + (size_t)j * blk, blk, cudaMemcpyHostToDevice,
                             d.stream));
    }
  }
  if (q8) {
    if (in16) f16_to_f32_kernel<<<1024, 256, 0, d.stream>>>((const f16*)st16, count, st32);
    int8_t* q = nullptr;
    if ((rc = dev_alloc(d, &q, count, err, errlen))) return rc;
    if ((rc = dev_alloc(d, &g.scale, (size_t)n, err, errlen))) return rc;
    quant_rows_kernel<<<std::min(4096, (n + 7) / 8), 256, 0, d.stream>>>(st32, n, k, q, g.scale);
    g.w = q;
  } else {
    if (!in16) f32_to_f16_kernel<<<1024, 256, 0, d.stream>>>(st32, count, w16);
    g.w = w16;
  }
  CU_TRY(cudaGetLastError());
  CU_TRY(cudaStreamSynchronize(d.stream));
  // Bias (interleaved like the weight for SwiGLU; an absent half is zero).
  if (b1 || b2) {
    std::vector<float> hb((size_t)n, 0.0f);
    if (!two) {
      memcpy(hb.data(), b1, sizeof(float) * n);
    } else {
      for (int j = 0; j * half < n1; ++j)
        for (int r = 0; r < half; ++r) {
          if (b1) hb[(size_t)2 * j * half + r] = b1[(size_t)j * half + r];
          if (b2) hb[(size_t)(2 * j + 1) * half + r] = b2[(size_t)j * half + r];
        }
    }
    if ((rc = upload_f32(d, &g.bias, hb.data(), (size_t)n, err, errlen))) return rc;
    CU_TRY(cudaStreamSynchronize(d.stream));  // hb is released on return
  }
  g.bn = two ? 2 * half : (ln_slices ? ln_slice_cols(n) : pick_bn(n));
  g.pair = !q8 && d.gemm_pair && g.bn <= 256;
  const uint32_t box = (g.pair || g.bn > 256) ? (uint32_t)g.bn / 2 : (uint32_t)g.bn;
  if (!make_operand_map(&g.map, g.w, q8 ? kElemS8 : kElemF16, (uint64_t)n, (uint64_t)k, box))
    return set_err(err, errlen, FUTON_ECUDA, "native: cuTensorMapEncodeTiled failed for a weight");
  return FUTON_OK;
}

// ---- workspace -----------------------------------------------------------
int ensure_workspace(const futon_model& m, DevCtx& d, size_t tokens, char* err, size_t errlen) {
  if (d.ws.tokens >= tokens) return FUTON_OK;
  if (d.ws.base) {
    CU_TRY(cudaDeviceSynchronize());  // callers may have queued work on their own stream
    cudaFree(d.ws.base);
    d.ws.base = nullptr;
    d.ws.tokens = 0;
  }
  const size_t T = tokens, h = m.cfg.hidden_size, I = m.cfg.intermediate_size;
  const bool q8 = m.q8 != 0;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes, 256); return o; };
  const size_t o_x = q8 ? take(T * h * 4) : 0, o_xb = q8 ? 0 : take(T * h * 2);
  const size_t o_xf = q8 ? 0 : take(T * h * 4);
  const size_t o_qkv = take(T * 3 * h * (q8 ? 4 : 2));
  const size_t o_attn = take(T * h * (q8 ? 4 : 2)), o_ffn = take(T * I * (q8 ? 4 : 2));
  const size_t o_tmp = (q8 || !m.fuse_ln) ? take(T * h * 4) : 0, o_xc = take(T * h * (q8 ? 4 : 2));
  size_t o_xq = 0, o_aq = 0, o_fq = 0, o_xs = 0, o_as = 0, o_fs = 0;
  if (q8) {
    o_xq = take(T * h); o_aq = take(T * h); o_fq = take(T * I);
    o_xs = take(T * 4); o_as = take(T * 4); o_fs = take(T * 4);
  }
  void* base = nullptr;
  CU_TRY(cudaMalloc(&base, off));
  uint8_t* b = static_cast<uint8_t*>(base);
  Workspace& w = d.ws;
  w.base = base;
  w.tokens = tokens;
  w.x = q8 ? (float*)(b + o_x) : nullptr;
  w.xb = q8 ? nullptr : (f16*)(b + o_xb);
  w.xf = q8 ? nullptr : (float*)(b + o_xf);
  w.qkv = b + o_qkv;
  w.attn = b + o_attn;
  w.ffn = b + o_ffn;
  w.tmp = (q8 || !m.fuse_ln) ? (float*)(b + o_tmp) : nullptr;
  w.xc = b + o_xc;
  w.xq = q8 ? (int8_t*)(b + o_xq) : nullptr;
  w.attnq = q8 ? (int8_t*)(b + o_aq) : nullptr;
  w.ffnq = q8 ? (int8_t*)(b + o_fq) : nullptr;
  w.xs = q8 ? (float*)(b + o_xs) : nullptr;
  w.attns = q8 ? (float*)(b + o_as) : nullptr;
  w.ffns = q8 ? (float*)(b + o_fs) : nullptr;
  return FUTON_OK;
}

template <typename T>
int ensure_dev(T** p, size_t* cap, size_t count, char* err, size_t errlen) {
  if (*cap >= count) return FUTON_OK;
  if (*p) {
    CU_TRY(cudaDeviceSynchronize());
    cudaFree(*p);
  }
  *p = nullptr;
  *cap = 0;
  size_t n = std::max<size_t>(count, 1024);
  CU_TRY(cudaMalloc((void**)p, n * sizeof(T)));
  *cap = n;
  return FUTON_OK;
}
template <typename T>
int ensure_host(T** p, size_t* cap, size_t count, char* err, size_t errlen) {
  if (*cap >= count) return FUTON_OK;
  if (*p) {
    CU_TRY(cudaDeviceSynchronize());
    cudaFreeHost(*p);
  }
  *p = nullptr;
  *cap = 0;
  size_t n = std::max<size_t>(count, 1024);
  CU_TRY(cudaMallocHost((void**)p, n * sizeof(T)));
  *cap = n;
  return FUTON_OK;
}

// ---- GEMM helper ---------------------------------------------------------
struct GemmOut {
  int epi = kEpiStore;
  bool out_f32 = false;
  void* out = nullptr;
  int ldo = 0;
  const void* resid = nullptr;
  int ldr = 0;
  bool resid_16 = false;  // the residual is f16 (else f32)
  const float* ln_w = nullptr;
  const float* ln_b = nullptr;
  float eps = 0.f;
  float* out_f32_copy = nullptr;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  int rope_hd = 0;
  int rope_cols = 0;
  const int* cu = nullptr;
  int nseq = 0;
  int f16_from = 1 << 30;
};

int run_gemm(DevCtx& d, int stage, const void* A, bool s8, const float* a_scale, int M,
             const GemmWeight& w, const GemmOut& o, cudaStream_t st, char* err, size_t errlen) {
  if (M == 0) return FUTON_OK;
  const double esz = s8 ? 1.0 : 2.0;
  const double out_cols = o.epi == kEpiSwiglu ? w.n / 2 : w.n;
  const bool plain = o.epi == kEpiStore || o.epi == kEpiRope;
  const double osz = (o.out_f32 || (s8 && !plain)) ? 4.0 : 2.0;
  const double rsz = o.resid ? (o.resid_16 ? 2.0 : 4.0) : 0.0;
  const double bytes = (double)M * w.k * esz + (double)w.n * w.k * esz + (double)M * out_cols * osz +
                       (double)M * w.n * rsz + (o.out_f32_copy ? (double)M * w.n * 4.0 : 0.0);
  ProfScope prof(d, st, stage, 2.0 * M * w.n * w.k, bytes);
  CUtensorMap ta, to;
  auto operand_map = [&](CUtensorMap* map, const void* base, bool is_s8, uint64_t rows,
                         uint64_t cols) {
    const Elem e = is_s8 ? kElemS8 : kElemF16;
    return d.map_cache.get(MapKey{kMapOperand, base, rows, cols, (uint64_t)e, 128}, map,
                           [&](CUtensorMap* mm) {
                             return make_operand_map(mm, base, e, rows, cols, 128);
                           });
  };
  if (!operand_map(&ta, A, s8, (uint64_t)M, (uint64_t)w.k))
    return set_err(err, errlen, FUTON_ECUDA, "native: cuTensorMapEncodeTiled failed (activation)");
  // 16-bit outputs leave through TMA tile stores.
  const bool out16 = o.epi == kEpiResidLN || !(o.out_f32 || (s8 && !plain));
  if (out16) {
    const uint64_t ncols = o.epi == kEpiSwiglu ? (uint64_t)w.n / 2 : (uint64_t)w.n;
    const MapKey key{kMapOutput, o.out, (uint64_t)M, ncols, (uint64_t)o.ldo, 0};
    if (!d.map_cache.get(key, &to, [&](CUtensorMap* mm) {
          return make_output_map(mm, o.out, (uint64_t)M, ncols, (uint64_t)o.ldo);
        }))
      return set_err(err, errlen, FUTON_ECUDA, "native: cuTensorMapEncodeTiled failed (output)");
  }
  CUtensorMap tr;
  if (o.epi == kEpiResidLN && !operand_map(&tr, o.resid, false, (uint64_t)M, (uint64_t)w.n))
    return set_err(err, errlen, FUTON_ECUDA, "native: cuTensorMapEncodeTiled failed (residual)");
  GemmLaunch g;
  g.ta = &ta;
  g.tw = &w.map;
  g.to = out16 ? &to : nullptr;
  g.tr = o.epi == kEpiResidLN ? &tr : nullptr;
  g.M = M;
  g.N = w.n;
  g.K = w.k;
  g.bn = w.bn;
  g.epi = o.epi;
  g.out_f32 = o.out_f32;
  g.f16 = !s8;
  g.pair = w.pair;
  g.pdl = d.pdl;
  g.ep.out = o.out;
  g.ep.ldo = o.ldo;
  g.ep.bias = w.bias;
  g.ep.resid = o.resid;
  g.ep.ldr = o.ldr;
  g.ep.resid_kind = o.resid_16 ? kResidF16 : kResidF32;
  g.ep.a_scale = a_scale;
  g.ep.w_scale = w.scale;
  g.ep.ln_w = o.ln_w;
  g.ep.ln_b = o.ln_b;
  g.ep.eps = o.eps;
  g.ep.out_f32 = o.out_f32_copy;
  g.ep.rope_cos = o.rope_cos;
  g.ep.rope_sin = o.rope_sin;
  g.ep.rope_hd = o.rope_hd;
  g.ep.rope_cols = o.rope_cols;
  g.ep.cu = o.cu;
  g.ep.nseq = o.nseq;
  g.ep.f16_from = o.f16_from;
  g.err = d.err_word;
  g.num_sms = d.num_sms;
  g.stream = st;
  cudaError_t e = s8 ? launch_gemm_s8(g) : launch_gemm_f16(g);
  if (e != cudaSuccess)
    return set_err(err, errlen, FUTON_ECUDA, "native: gemm launch: %s", cudaGetErrorString(e));
  d.launches.fetch_add(1, std::memory_order_relaxed);
  return FUTON_OK;
}

// Kernel launch on st; with pdl the kernel may start while the kernel before
// it in the stream finishes (programmatic dependent launch: the kernels of
// the forward wait for their predecessor with pdl_wait before they touch
// global memory).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t st, Args&&... args) {
  if (!pdl) {
    kern<<<grid, block, smem, st>>>(std::forward<Args>(args)...);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

inline int grid_rows(int rows, int per_block, int sms) {
  long g = (rows + per_block - 1) / per_block;
  long cap = (long)sms * 16;
  return (int)std::max<long>(1, std::min(g, cap));
}

// ---- attention dispatch --------------------------------------------------
// attn_tc2_kernel (tcgen05, packed 128-row windows) is parity-correct and
// batch-invariant but, as measured on the c4 workload, 1.4× slower than
// attn_heads_kernel; it runs only when FUTON_CUDA_ATTN=tc2.
enum AttnKind : int { kAttnHeads = 0, kAttnTc2 = 2 };

// Model-creation-time attention options from the environment; unknown
// values leave the defaults.
void read_attn_env(futon_model& m) {
  if (const char* v = std::getenv("FUTON_CUDA_ATTN")) {
    if (!strcmp(v, "tc2")) m.attn_kind = kAttnTc2;
    else if (!strcmp(v, "heads")) m.attn_kind = kAttnHeads;
  }
  if (const char* v = std::getenv("FUTON_CUDA_ATTN_SPLIT")) {
    if (!strcmp(v, "0")) m.attn_split = false;
    else if (!strcmp(v, "1")) m.attn_split = true;
  }
  if (const char* v = std::getenv("FUTON_CUDA_Q8_ATTN")) {
    if (!strcmp(v, "split")) m.q8_exact_attn = false;
    else if (!strcmp(v, "exact")) m.q8_exact_attn = true;
  }
  if (const char* v = std::getenv("FUTON_CUDA_GEMM_PAIR")) {
    if (!strcmp(v, "1")) m.gemm_pair = true;
    else if (!strcmp(v, "0")) m.gemm_pair = false;
  }
}

// CTAs per tile (grid.y) for attn_heads_kernel's head-group split: enough to
// give every SM about two CTAs, at most one per head group.
int attn_split_ways(const futon_model& m, const DevCtx& d, int tiles, int ngroups) {
  if (!m.attn_split || tiles <= 0 || ngroups <= 1) return 1;
  const int want = (2 * d.num_sms + tiles - 1) / tiles;
  return std::max(1, std::min(ngroups, want));
}

// A micro-batch's attention work lists (device memory): 64-query tiles per
// sequence and ≤ 128-row windows of packed sequences.
struct AttnPlan {
  const AttnTile* tiles;
  int ntiles;
  const AttnTile* cls_tiles;  // one (sequence, 0) per sequence, longest first
  const AttnWindow* wins;
  int nwin;
  const AttnSeg* segs;
  // Exact int8-path attention: per-sequence offsets of P (all query rows /
  // the CLS row only), their totals, the scratch and heads per launch.
  const int* poff = nullptr;
  const int* pcls = nullptr;
  size_t ptot = 0, ptot_cls = 0;
  float* pscr = nullptr;
  int head_group = 0;
  // float32(1/Σe) per (head of the group, query row or CLS sequence).
  float* pinv = nullptr;
  int pinv_ld = 0;
};

// q and k arrive already rotated (RoPE runs in the qkv GEMM epilogue).
// Float path: f16 qkv, attn_heads_kernel (one CTA per 64-query tile, or per
// sequence for the CLS-only last layer). Int8 path: f32 qkv and split-precision attention,
// so the per-row quantisation that follows sees float32-accurate values.
// Head dims other than 32/64 use the per-query kernel.
template <typename InT, typename OutT>
int run_attention(const futon_model& m, DevCtx& d, int T, int nseq, const int* cu,
                  const AttnPlan& plan, bool cls_only, const InT* qkv, OutT* out,
                  cudaStream_t st, char* err, size_t errlen) {
  const int h = m.cfg.hidden_size, H = m.cfg.num_heads, hd = m.head_dim;
  const float scale_log2 = (float)(1.0 / std::sqrt((double)hd) * 1.4426950408889634);
  constexpr bool kSplit = sizeof(InT) == 4;
  const bool tc_hd = hd == 32 || hd == 64;
  // The CLS-only layer walks its own list: (sequence, query 0), longest first.
  const AttnTile* tiles = cls_only ? plan.cls_tiles : plan.tiles;
  const int ntiles = plan.ntiles;
  if constexpr (!kSplit) {
    if (m.attn_kind == kAttnTc2 && tc_hd && H % 2 == 0 && !cls_only) {
      if (plan.nwin == 0) return FUTON_OK;
      // 64-column q, k, v tiles (a head pair for head_dim 32, a head for 64):
      // 16·n rows, 128-byte swizzle.
      AttnMaps maps{};
      for (int n = 1; n <= 8; ++n)
        if (!d.map_cache.get(MapKey{kMapQkv, qkv, (uint64_t)T, (uint64_t)(3 * h), 64u, 16u * n},
                             &maps.m[n], [&](CUtensorMap* mm) {
                               return make_qkv_map(mm, qkv, (uint64_t)T, (uint64_t)(3 * h), 64,
                                                   16u * n);
                             }))
          return set_err(err, errlen, FUTON_ECUDA, "native: cuTensorMapEncodeTiled failed (qkv)");
      const int smem = attn_tc2_smem_bytes();
      auto launch = [&](auto kern) -> cudaError_t {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        kern<<<plan.nwin, AttnTc2Cfg::kThreads, smem, st>>>(maps, h, H, plan.wins, plan.segs,
                                                             scale_log2, out, h, d.err_word);
        return cudaGetLastError();
      };
      CU_TRY(hd == 32 ? launch(attn_tc2_kernel<32, OutT>) : launch(attn_tc2_kernel<64, OutT>));
      d.launches.fetch_add(1, std::memory_order_relaxed);
      return FUTON_OK;
    }
    if (tc_hd) {
      const int grid = cls_only ? nseq : ntiles;
      if (grid == 0) return FUTON_OK;
      // q, k, v tiles of nh adjacent heads: 64 rows × nh·hd columns, swizzled
      // over one row.
      const int nh = attn_heads_per_step(hd, H);
      CUtensorMap tm;
      if (!d.map_cache.get(MapKey{kMapQkv, qkv, (uint64_t)T, (uint64_t)(3 * h),
                                  (uint64_t)(nh * hd), 64},
                           &tm, [&](CUtensorMap* mm) {
                             return make_qkv_map(mm, qkv, (uint64_t)T, (uint64_t)(3 * h), nh * hd,
                                                 64);
                           }))
        return set_err(err, errlen, FUTON_ECUDA, "native: cuTensorMapEncodeTiled failed (qkv)");
      const int ways = attn_split_ways(m, d, grid, H / nh);
      auto launch = [&](auto kern, int smem) -> cudaError_t {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        return launch_k(d.pdl, kern, dim3(grid, ways), dim3(128), (size_t)smem, st, tm, h, H, cu,
                        tiles, cls_only ? 1 : 0, scale_log2, out, h, d.err_word);
      };
      if (ways > 1)
        CU_TRY(hd == 64   ? launch(attn_heads_kernel<64, 1, OutT, true>, attn_heads_smem_bytes<64, 1>())
               : nh == 2 ? launch(attn_heads_kernel<32, 2, OutT, true>, attn_heads_smem_bytes<32, 2>())
                         : launch(attn_heads_kernel<32, 1, OutT, true>, attn_heads_smem_bytes<32, 1>()));
      else
        CU_TRY(hd == 64   ? launch(attn_heads_kernel<64, 1, OutT>, attn_heads_smem_bytes<64, 1>())
               : nh == 2 ? launch(attn_heads_kernel<32, 2, OutT>, attn_heads_smem_bytes<32, 2>())
                         : launch(attn_heads_kernel<32, 1, OutT>, attn_heads_smem_bytes<32, 1>()));
      d.launches.fetch_add(1, std::memory_order_relaxed);
      return FUTON_OK;
    }
  } else {
    if (plan.pscr && tc_hd) {
      // Exact operation order (attn_exact.cuh), head groups of plan.head_group.
      const int grid = cls_only ? nseq : ntiles;
      if (grid == 0) return FUTON_OK;
      const int* poff = cls_only ? plan.pcls : plan.poff;
      const size_t pstride = cls_only ? plan.ptot_cls : plan.ptot;
      const float scale = (float)(1.0 / std::sqrt((double)hd));
      const int cls = cls_only ? 1 : 0;
      for (int h0 = 0; h0 < H; h0 += plan.head_group) {
        const unsigned nh = (unsigned)std::min(plan.head_group, H - h0);
        if (hd == 32) {
          attn_exact_softmax_kernel<32><<<dim3(grid, nh), 64, 0, st>>>(
              qkv, h, h0, cu, tiles, cls, poff, pstride, scale, plan.pscr, plan.pinv, plan.pinv_ld);
          attn_exact_pv_kernel<32><<<dim3(grid, 2, nh), 4 * 32, 0, st>>>(
              qkv, h, h0, cu, tiles, cls, poff, pstride, plan.pscr, plan.pinv, plan.pinv_ld, out, h);
        } else {
          attn_exact_softmax_kernel<64><<<dim3(grid, nh), 64, 0, st>>>(
              qkv, h, h0, cu, tiles, cls, poff, pstride, scale, plan.pscr, plan.pinv, plan.pinv_ld);
          attn_exact_pv_kernel<64><<<dim3(grid, 2, nh), 4 * 64, 0, st>>>(
              qkv, h, h0, cu, tiles, cls, poff, pstride, plan.pscr, plan.pinv, plan.pinv_ld, out, h);
        }
        CU_TRY(cudaGetLastError());
        d.launches.fetch_add(2, std::memory_order_relaxed);
      }
      return FUTON_OK;
    }
    if (tc_hd && !cls_only && ntiles > 0) {
      dim3 grid(ntiles, H);
      const int smem = 6 * 64 * (hd + 8) * 2;
      auto launch = [&](auto kern) -> cudaError_t {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        kern<<<grid, 128, smem, st>>>(qkv, h, cu, tiles, nullptr, nullptr, scale_log2, out, h);
        return cudaGetLastError();
      };
      CU_TRY(hd == 32 ? launch(attn_flash_split_kernel<32, false>)
                      : launch(attn_flash_split_kernel<64, false>));
      d.launches.fetch_add(1, std::memory_order_relaxed);
      return FUTON_OK;
    }
  }
  const int nq = cls_only ? nseq : T;
  const long warps = (long)nq * H;
  const int blocks = (int)((warps * 32 + 255) / 256);
  if (blocks == 0) return FUTON_OK;
#define FUTON_ROWQ(HD_)                                                                   \
  launch_k(d.pdl, attn_rowq_kernel<HD_, InT, OutT>, dim3(blocks), dim3(256), 0, st, qkv, h, H, \
           cu, nseq, nq, cls_only ? 1 : 0, (const float*)nullptr, (const float*)nullptr, 0,  \
           scale_log2, out, h)
  switch (hd) {
    case 8: FUTON_ROWQ(8); break;
    case 16: FUTON_ROWQ(16); break;
    case 32: FUTON_ROWQ(32); break;
    case 64: FUTON_ROWQ(64); break;
    default: return set_err(err, errlen, FUTON_EINVAL, "native: unsupported head_dim %d", hd);
  }
#undef FUTON_ROWQ
  CU_TRY(cudaGetLastError());
  d.launches.fetch_add(1, std::memory_order_relaxed);
  return FUTON_OK;
}

// ---- one micro-batch -----------------------------------------------------
// ids: device [T]; cu: device [nseq+1] (local offsets); tiles: device.
// sum_l2 = Σ L² over the micro-batch's sequences (attention work, profiler only).
int forward_mb(const futon_model& m, DevCtx& d, const int* ids, const int* cu, int nseq, int T,
               double sum_l2, const AttnPlan& plan, int out_dim, float* out,
               cudaStream_t st, volatile const int* cancel, char* err, size_t errlen) {
  const futon_cfg& c = m.cfg;
  const int h = c.hidden_size, I = c.intermediate_size;
  const bool q8 = m.q8 != 0, cls = c.pooling == FUTON_POOL_CLS;
  const float eps = (float)c.layer_norm_eps;
  Workspace& w = d.ws;
  int rc;

  {
    const double pos_bytes = c.position_encoding == FUTON_POS_ABSOLUTE ? 4.0 * h : 0.0;
    const double out_bytes = q8 ? 5.0 * h : 2.0 * h;
    ProfScope prof(d, st, kStEmbed, 0.0, (double)T * (4.0 + 4.0 * h + pos_bytes + out_bytes));
    if (q8 && m.q8_exact_attn)
      embed_ln_kernel<true><<<grid_rows(T, 8, d.num_sms), 256, 0, st>>>(
          ids, cu, nseq, T, h, c.vocab_size, d.err_word, d.word, d.type0, d.pos, d.embw, d.embb,
          eps, w.x, w.xb, w.xq, w.xs);
    else
      CU_TRY(launch_k(d.pdl, embed_ln_kernel<false>, dim3(grid_rows(T, 8, d.num_sms)), dim3(256),
                      0, st, ids, cu, nseq, T, h, c.vocab_size, d.err_word, d.word, d.type0,
                      d.pos, d.embw, d.embb, eps, w.x, w.xb, w.xq, w.xs));
    CU_TRY(cudaGetLastError());
    d.launches.fetch_add(1, std::memory_order_relaxed);
  }

  for (int li = 0; li < c.num_layers; ++li) {
    if (canceled(cancel))
      return set_err(err, errlen, FUTON_ECANCELED, "native: context canceled");
    const LayerDev& L = d.layers[li];
    const bool last = li == c.num_layers - 1;
    const bool last_cls = cls && last;
    const int rows = last_cls ? nseq : T;

    // qkv = x·Wqkvᵀ + b → [T, 3h] (f16 on the float path, f32 on the int8
    // path)
    {
      GemmOut o;
      o.epi = kEpiStore;
      o.out_f32 = q8;
      o.out = w.qkv;
      o.ldo = 3 * h;
      if (c.position_encoding == FUTON_POS_ROPE) {
        o.epi = kEpiRope;
        o.rope_cos = d.rcos;
        o.rope_sin = d.rsin;
        o.rope_hd = m.head_dim;
        o.rope_cols = 2 * h;
        o.cu = cu;
        o.nseq = nseq;
      }
      if ((rc = run_gemm(d, kStGemmQkv, q8 ? (const void*)w.xq : w.xb, q8, w.xs, T, L.qkv, o, st,
                         err, errlen)))
        return rc;
    }

    // attention → attn [rows, h]
    {
      const double esz = q8 ? 4.0 : 2.0;
      const double fl = last_cls ? 4.0 * (double)T * h : 4.0 * sum_l2 * h;
      const double by = (double)T * 3.0 * h * esz + (double)rows * h * esz;
      ProfScope prof(d, st, last_cls ? kStAttnCls : kStAttn, fl, by);
      if (q8)
        rc = run_attention<float, float>(m, d, T, nseq, cu, plan, last_cls,
                                         (const float*)w.qkv, (float*)w.attn, st, err, errlen);
      else
        rc = run_attention<f16, f16>(m, d, T, nseq, cu, plan, last_cls,
                                     (const f16*)w.qkv, (f16*)w.attn, st, err, errlen);
      if (rc) return rc;
    }

    // Residual stream rows for this layer's query side.
    const void* resid = q8 ? (const void*)w.x : (const void*)w.xb;
    if (last_cls) {
      const size_t esz = q8 ? 4 : 2;
      ProfScope prof(d, st, kStGather, 0.0, (double)nseq * 2.0 * h * esz);
      const int blocks = grid_rows((int)((size_t)nseq * h * esz / 16), 256, d.num_sms);
      if (q8) gather_rows_kernel<float><<<blocks, 256, 0, st>>>(w.x, cu, nseq, h, (float*)w.xc);
      else CU_TRY(launch_k(d.pdl, gather_rows_kernel<f16>, dim3(blocks), dim3(256), 0, st,
                           (const f16*)w.xb, cu, nseq, h, (f16*)w.xc));
      CU_TRY(cudaGetLastError());
      d.launches.fetch_add(1, std::memory_order_relaxed);
      resid = w.xc;
    }

    // Residual block: out = LN(x + W·a + b), written over the residual stream.
    auto resid_ln = [&](int stage, const void* A, const float* a_scale, const GemmWeight& W,
                        const void* res, const float* lnw, const float* lnb,
                        bool f32_copy) -> int {
      GemmOut o;
      if (m.fuse_ln) {
        o.epi = kEpiResidLN;
        o.out = w.xb;
        o.ldo = h;
        o.resid = res;
        o.ldr = h;
        o.resid_16 = true;
        o.ln_w = lnw;
        o.ln_b = lnb;
        o.eps = eps;
        o.out_f32_copy = f32_copy ? w.xf : nullptr;
        return run_gemm(d, stage, A, q8, a_scale, rows, W, o, st, err, errlen);
      }
      o.epi = kEpiResid;
      o.out_f32 = true;
      o.out = w.tmp;
      o.ldo = h;
      o.resid = res;
      o.ldr = h;
      o.resid_16 = !q8;
      int r2 = run_gemm(d, stage, A, q8, a_scale, rows, W, o, st, err, errlen);
      if (r2) return r2;
      ProfScope prof(d, st, kStLayerNorm, 0.0, (double)rows * h * (q8 ? 9.0 : (f32_copy ? 10.0 : 6.0)));
      float* xo = q8 ? w.x : (f32_copy ? w.xf : nullptr);
      if (q8 && m.q8_exact_attn)
        layernorm_kernel<true><<<grid_rows(rows, 256, d.num_sms), 256, 0, st>>>(
            w.tmp, rows, h, lnw, lnb, eps, xo, nullptr, w.xq, w.xs);
      else
        CU_TRY(launch_k(d.pdl, layernorm_kernel<false>, dim3(grid_rows(rows, 8, d.num_sms)),
                        dim3(256), 0, st, (const float*)w.tmp, rows, h, lnw, lnb, eps, xo,
                        q8 ? nullptr : w.xb, w.xq, w.xs));
      CU_TRY(cudaGetLastError());
      d.launches.fetch_add(1, std::memory_order_relaxed);
      return FUTON_OK;
    };

    // out projection + residual + LN1
    const void* a_out = w.attn;
    const float* a_out_s = nullptr;
    if (q8) {
      ProfScope prof(d, st, kStQuant, 0.0, (double)rows * h * 5.0 + rows * 4.0);
      quant_rows_kernel<<<grid_rows(rows, 8, d.num_sms), 256, 0, st>>>((const float*)w.attn, rows,
                                                                     h, w.attnq, w.attns);
      CU_TRY(cudaGetLastError());
      d.launches.fetch_add(1, std::memory_order_relaxed);
      a_out = w.attnq;
      a_out_s = w.attns;
    }
    if ((rc = resid_ln(kStGemmOut, a_out, a_out_s, L.out, resid, L.n1w, L.n1b, false))) return rc;

    if (canceled(cancel))
      return set_err(err, errlen, FUTON_ECANCELED, "native: context canceled");

    // FFN
    {
      GemmOut o;
      o.epi = c.activation == FUTON_ACT_SWIGLU ? kEpiSwiglu : kEpiGelu;
      o.out_f32 = q8;
      o.out = w.ffn;
      o.ldo = I;
      if ((rc = run_gemm(d, kStGemmFc1, q8 ? (const void*)w.xq : w.xb, q8, w.xs, rows, L.fc1, o, st,
                         err, errlen)))
        return rc;
    }
    const void* a_fc2 = w.ffn;
    const float* a_fc2_s = nullptr;
    if (q8) {
      ProfScope prof(d, st, kStQuant, 0.0, (double)rows * I * 5.0 + rows * 4.0);
      quant_rows_kernel<<<grid_rows(rows, 8, d.num_sms), 256, 0, st>>>((const float*)w.ffn, rows, I,
                                                                     w.ffnq, w.ffns);
      CU_TRY(cudaGetLastError());
      d.launches.fetch_add(1, std::memory_order_relaxed);
      a_fc2 = w.ffnq;
      a_fc2_s = w.ffns;
    }
    const void* resid2 = q8 ? (const void*)w.x : (const void*)w.xb;
    if ((rc = resid_ln(kStGemmFc2, a_fc2, a_fc2_s, L.fc2, resid2, L.n2w, L.n2b, last))) return rc;
  }

  {
    const int dim = out_dim ? out_dim : h;
    const double rows_read = cls ? (double)nseq : (double)T;
    ProfScope prof(d, st, kStPool, 0.0, rows_read * h * 4.0 + (double)nseq * dim * 4.0);
    const int mat_ln = c.matryoshka_layernorm ? 1 : 0;
    CU_TRY(launch_k(d.pdl, pool_kernel, dim3(nseq), dim3(256), h * sizeof(float), st,
                    (const float*)(q8 ? w.x : w.xf), cu, h, cls ? 0 : 1, out_dim, mat_ln,
                    c.normalize ? 1 : 0, out));
    CU_TRY(cudaGetLastError());
    d.launches.fetch_add(1, std::memory_order_relaxed);
  }
  return FUTON_OK;
}

// ---- call planning -------------------------------------------------------
struct MicroBatch {
  int s0, s1;   // sequences [s0, s1)
  int t0, t1;   // tokens [t0, t1)
  size_t cu_off, tile_off, cls_off, win_off, seg_off;  // int offsets into the meta buffer
  int ntiles, nwin, nseg;
  double sum_l2;            // Σ L² (profiler)
  // Exact int8-path attention: offsets of the P row blocks (meta) and totals.
  size_t poff_off = 0, pcls_off = 0;
  size_t ptot = 0, ptot_cls = 0;
};

// Attention windows of sequences [s0, s1) (token offsets relative to t0):
// sequences of ≤ 128 tokens are packed whole, in order, into windows, each
// at the next 16-row boundary, while the rows fit in 128; a longer sequence
// gets one window per 128 queries, keyed by the whole sequence. Writes
// `wins` / `segs` when given; returns the window count and adds the segment
// count to *nsegs.
int plan_windows(const int32_t* cu, int s0, int s1, int t0, AttnWindow* wins, AttnSeg* segs,
                 int* nsegs) {
  int n = 0, ns = 0;
  int open = -1;  // window still accepting short sequences
  int used = 0;   // its rows
  for (int s = s0; s < s1; ++s) {
    const int a = cu[s] - t0, L = cu[s + 1] - cu[s];
    if (L <= 128) {
      const int pad = (L + 15) & ~15;
      if (open < 0 || used + pad > 128) {
        if (wins) wins[n] = AttnWindow{0, 0, 0, 0, ns, 0};
        open = n++;
        used = 0;
      }
      if (segs) segs[ns] = AttnSeg{a, L, used};
      ++ns;
      used += pad;
      if (wins) {
        wins[open].nq = wins[open].nk = used;
        wins[open].nseg += 1;
      }
    } else {
      open = -1;
      for (int q = a; q < a + L; q += 128) {
        if (wins) wins[n] = AttnWindow{q, std::min(128, a + L - q), a, L, 0, 0};
        ++n;
      }
    }
  }
  *nsegs += ns;
  return n;
}

int validate_input(const futon_model& m, const int32_t* cu, int nseq, int out_dim, char* err,
                   size_t errlen) {
  const futon_cfg& c = m.cfg;
  if (nseq < 0) return set_err(err, errlen, FUTON_EINVAL, "native: negative sequence count");
  if (nseq > 0 && !cu) return set_err(err, errlen, FUTON_EINVAL, "native: null cu_seqlens");
  if (out_dim < 0 || out_dim > c.hidden_size)
    return set_err(err, errlen, FUTON_EINVAL, "native: requested dim %d outside [1,%d]", out_dim,
                   c.hidden_size);
  if (out_dim != 0 && out_dim != c.hidden_size && !c.matryoshka)
    return set_err(err, errlen, FUTON_EINVAL,
                   "native: pack does not support matryoshka truncation to %d", out_dim);
  if (nseq > 0 && cu[0] != 0)
    return set_err(err, errlen, FUTON_EINVAL, "native: cu_seqlens[0] must be 0");
  for (int s = 0; s < nseq; ++s) {
    const int L = cu[s + 1] - cu[s];
    if (L <= 0) return set_err(err, errlen, FUTON_EINVAL, "native: batch item %d: empty token sequence", s);
    if (L > m.eff_max)
      return set_err(err, errlen, FUTON_EINVAL,
                     "native: batch item %d: sequence length %d exceeds effective max_seq_len %d", s,
                     L, m.eff_max);
  }
  return FUTON_OK;
}

// Every id in [0, vocab): one branch-free pass over the packed ids (cu is
// validated, so they are exactly [0, cu[nseq])); the first bad id and its
// sequence are looked up only when there is one.
int check_ids(const futon_model& m, const int32_t* ids, const int32_t* cu, int nseq, char* err,
              size_t errlen) {
  const uint32_t V = (uint32_t)m.cfg.vocab_size;
  const size_t T = nseq > 0 ? (size_t)cu[nseq] : 0;
  uint32_t bad = 0;
  for (size_t t = 0; t < T; ++t) bad |= (uint32_t)((uint32_t)ids[t] >= V);
  if (!bad) return FUTON_OK;
  size_t t = 0;
  while ((uint32_t)ids[t] < V) ++t;
  const int s = (int)(std::upper_bound(cu, cu + nseq + 1, (int32_t)t) - cu) - 1;
  return set_err(err, errlen, FUTON_EINVAL, "native: batch item %d: token id %d outside vocab of %d",
                 s, ids[t], (int)V);
}

// Splits a call into micro-batches and lays out their metadata in the
// pinned meta buffer (offsets only; upload_mb_meta fills and uploads each
// one just before its forward, so the host plans micro-batch i + 1 while the
// GPU runs i). windows: the tcgen05 attention's window lists are planned too.
int plan_batches(DevCtx& d, const int32_t* cu, int nseq, bool exact_p, bool windows,
                 std::vector<MicroBatch>& mbs, char* err, size_t errlen) {
  mbs.clear();
  size_t meta = 0;
  for (int s = 0; s < nseq;) {
    MicroBatch mb;
    mb.s0 = s;
    mb.t0 = cu[s];
    int ntiles = 0;
    double l2 = 0.0;
    size_t pacc = 0;  // exact_p: Σ pad8(L)·L so far
    while (s < nseq && (s == mb.s0 || cu[s + 1] - mb.t0 <= kTokenBudget)) {
      const size_t Lz = (size_t)(cu[s + 1] - cu[s]);
      if (exact_p && s > mb.s0 && pacc + ((Lz + 7) & ~(size_t)7) * Lz > kExactPBudget) break;
      pacc += ((Lz + 7) & ~(size_t)7) * Lz;
      const double Ls = cu[s + 1] - cu[s];
      ntiles += (cu[s + 1] - cu[s] + 63) / 64;
      l2 += Ls * Ls;
      ++s;
    }
    mb.sum_l2 = l2;
    mb.s1 = s;
    mb.t1 = cu[s];
    mb.ntiles = ntiles;
    mb.nseg = 0;
    mb.nwin = windows ? plan_windows(cu, mb.s0, mb.s1, mb.t0, nullptr, nullptr, &mb.nseg) : 0;
    mb.cu_off = meta;
    meta += align_up((size_t)(mb.s1 - mb.s0 + 1), 4);
    mb.tile_off = meta;
    meta += align_up((size_t)ntiles * 2, 4);
    mb.cls_off = meta;
    meta += align_up((size_t)(mb.s1 - mb.s0) * 2, 4);
    mb.win_off = meta;
    meta += align_up((size_t)mb.nwin * 6, 4);
    mb.seg_off = meta;
    meta += align_up((size_t)mb.nseg * 3, 4);
    if (exact_p) {
      // P holds pad8(L) keys × L query rows per sequence (1 row for the CLS
      // layer); offsets are int, so a micro-batch's total must fit in one.
      for (int q = mb.s0; q < mb.s1; ++q) {
        const size_t L = (size_t)(cu[q + 1] - cu[q]), kp = (L + 7) & ~(size_t)7;
        mb.ptot += kp * L;
        mb.ptot_cls += kp;
      }
      if (mb.ptot > (size_t)INT32_MAX)
        return set_err(err, errlen, FUTON_EINVAL,
                       "native: micro-batch too large for the exact int8 attention");
      mb.poff_off = meta;
      meta += align_up((size_t)(mb.s1 - mb.s0 + 1), 4);
      mb.pcls_off = meta;
      meta += align_up((size_t)(mb.s1 - mb.s0 + 1), 4);
    }
    mbs.push_back(mb);
  }
  if (mbs.empty()) return FUTON_OK;
  // The pinned staging may still feed the previous call's uploads.
  CU_TRY(cudaEventSynchronize(d.meta_evt));
  int rc;
  if ((rc = ensure_host(&d.h_meta, &d.h_meta_cap, meta, err, errlen))) return rc;
  if ((rc = ensure_dev(&d.d_meta, &d.d_meta_cap, meta, err, errlen))) return rc;
  return FUTON_OK;
}

// Fills micro-batch mb's metadata (local cu_seqlens, attention tiles and
// CLS list longest sequence first, tcgen05 windows when planned, the exact
// int8 attention's P offsets) and uploads it on st.
int upload_mb_meta(DevCtx& d, const int32_t* cu, const MicroBatch& mb, bool exact_p, bool windows,
                   cudaStream_t st, char* err, size_t errlen) {
  int* hc = d.h_meta + mb.cu_off;
  int maxL = 0;
  for (int s = mb.s0; s <= mb.s1; ++s) hc[s - mb.s0] = cu[s] - mb.t0;
  for (int s = mb.s0; s < mb.s1; ++s) maxL = std::max(maxL, cu[s + 1] - cu[s]);
  // Tiles longest sequence first (the CTAs launch in list order, so the
  // tiles with the most key blocks start early instead of trailing the
  // launch); every tile is computed the same way in any order. A counting
  // sort on the length, ties in sequence order: the order a stable sort by
  // decreasing length gives. slot[L]: next free entry for length L.
  std::vector<int>& slot = d.plan_slots;
  auto order = [&](int per_tile) {
    slot.assign((size_t)maxL + 1, 0);
    for (int s = mb.s0; s < mb.s1; ++s) {
      const int L = cu[s + 1] - cu[s];
      slot[L] += per_tile ? (L + 63) / 64 : 1;
    }
    int acc = 0;
    for (int L = maxL; L >= 0; --L) {
      const int c = slot[L];
      slot[L] = acc;
      acc += c;
    }
  };
  AttnTile* ht = reinterpret_cast<AttnTile*>(d.h_meta + mb.tile_off);
  order(1);
  for (int s = mb.s0; s < mb.s1; ++s) {
    const int L = cu[s + 1] - cu[s];
    for (int q0 = 0; q0 < L; q0 += 64) ht[slot[L]++] = AttnTile{s - mb.s0, q0};
  }
  // The CLS-only last layer: one query row per sequence, same order.
  AttnTile* hcl = reinterpret_cast<AttnTile*>(d.h_meta + mb.cls_off);
  order(0);
  for (int s = mb.s0; s < mb.s1; ++s) hcl[slot[cu[s + 1] - cu[s]]++] = AttnTile{s - mb.s0, 0};
  if (windows) {
    int nseg = 0;
    AttnWindow* hw = reinterpret_cast<AttnWindow*>(d.h_meta + mb.win_off);
    plan_windows(cu, mb.s0, mb.s1, mb.t0, hw, reinterpret_cast<AttnSeg*>(d.h_meta + mb.seg_off),
                 &nseg);
    // tcgen05 windows most keys first (each keeps its own segment range).
    std::stable_sort(hw, hw + mb.nwin,
                     [](const AttnWindow& a, const AttnWindow& b) { return a.nk > b.nk; });
  }
  if (exact_p) {
    int* po = d.h_meta + mb.poff_off;
    int* pc = d.h_meta + mb.pcls_off;
    po[0] = pc[0] = 0;
    for (int q = mb.s0; q < mb.s1; ++q) {
      const int L = cu[q + 1] - cu[q], kp = (L + 7) & ~7;
      po[q - mb.s0 + 1] = po[q - mb.s0] + kp * L;
      pc[q - mb.s0 + 1] = pc[q - mb.s0] + kp;
    }
  }
  // The micro-batch's block of the meta buffer: from its cu list to the end
  // of its last list (the layout is contiguous per micro-batch).
  const size_t lo = mb.cu_off;
  const size_t hi = exact_p ? mb.pcls_off + align_up((size_t)(mb.s1 - mb.s0 + 1), 4)
                            : mb.seg_off + align_up((size_t)mb.nseg * 3, 4);
  CU_TRY(cudaMemcpyAsync(d.d_meta + lo, d.h_meta + lo, (hi - lo) * sizeof(int),
                         cudaMemcpyHostToDevice, st));
  d.h2d_bytes.fetch_add((long long)((hi - lo) * sizeof(int)), std::memory_order_relaxed);
  CU_TRY(cudaEventRecord(d.meta_evt, st));
  return FUTON_OK;
}

// after_mb (optional) runs after each micro-batch's forward is queued, with
// the micro-batch's index and its sequences [s0, s1).
// before_mb (optional) runs after the micro-batch's metadata upload is
// queued and before its forward, with its index and tokens [t0, t1).
using MbHook = std::function<int(int, int, int)>;

// Calls of one micro-batch of at most this many tokens run from a CUDA graph
// when allow_graph is set (the host-buffer entry point, whose buffers are the
// library's own): launch-bound sizes, where ~60 kernel launches per forward
// cost as much as the kernels.
constexpr int kGraphMaxTokens = 32768;
constexpr size_t kGraphCacheSize = 32;

int run_call(const futon_model& m, DevCtx& d, const int* d_ids, const int32_t* cu, int nseq,
             int out_dim, float* d_out, cudaStream_t st, volatile const int* cancel, char* err,
             size_t errlen, const MbHook& after_mb = nullptr, const MbHook& before_mb = nullptr,
             bool allow_graph = false) {
  // Work of earlier calls (possibly on other streams) finishes before this
  // call's uploads and kernels touch the shared buffers; this call's end is
  // recorded for the next one on every return path.
  CU_TRY(cudaStreamWaitEvent(st, d.done_evt, 0));
  struct RecordDone {
    DevCtx& d;
    cudaStream_t st;
    ~RecordDone() { cudaEventRecord(d.done_evt, st); }
  } record_done{d, st};
  std::vector<MicroBatch> mbs;
  int rc;
  const bool exact_p = m.q8 && m.q8_exact_attn && (m.head_dim == 32 || m.head_dim == 64);
  const bool windows = m.attn_kind == kAttnTc2 && !m.q8;
  if ((rc = plan_batches(d, cu, nseq, exact_p, windows, mbs, err, errlen))) return rc;
  size_t max_t = 0, max_p = 0;
  for (const MicroBatch& mb : mbs) {
    max_t = std::max<size_t>(max_t, (size_t)(mb.t1 - mb.t0));
    max_p = std::max(max_p, mb.ptot);
  }
  if ((rc = ensure_workspace(m, d, max_t, err, errlen))) return rc;
  // Exact attention scratch: as many heads per launch as fit in 4 GiB of P,
  // then each head's per-row 1/Σe (max_t rows: every micro-batch's query
  // rows and CLS sequences fit).
  int head_group = 0;
  if (exact_p && max_p > 0) {
    const size_t budget = kExactPBudget;  // floats
    head_group = (int)std::max<size_t>(1, std::min<size_t>((size_t)m.cfg.num_heads, budget / max_p));
    if ((rc = ensure_dev(&d.d_pscr, &d.d_pscr_cap, (size_t)head_group * (max_p + max_t), err,
                         errlen)))
      return rc;
  }
  const int dim = out_dim ? out_dim : m.cfg.hidden_size;
  for (size_t i = 0; i < mbs.size(); ++i) {
    const MicroBatch& mb = mbs[i];
    if (canceled(cancel))
      return set_err(err, errlen, FUTON_ECANCELED, "native: context canceled");
    if ((rc = upload_mb_meta(d, cu, mb, exact_p, windows, st, err, errlen))) return rc;
    if (before_mb && (rc = before_mb((int)i, mb.t0, mb.t1))) return rc;
    AttnPlan plan{reinterpret_cast<const AttnTile*>(d.d_meta + mb.tile_off), mb.ntiles,
                  reinterpret_cast<const AttnTile*>(d.d_meta + mb.cls_off),
                  reinterpret_cast<const AttnWindow*>(d.d_meta + mb.win_off), mb.nwin,
                  reinterpret_cast<const AttnSeg*>(d.d_meta + mb.seg_off)};
    if (head_group > 0) {
      plan.poff = d.d_meta + mb.poff_off;
      plan.pcls = d.d_meta + mb.pcls_off;
      plan.ptot = mb.ptot;
      plan.ptot_cls = mb.ptot_cls;
      plan.pscr = d.d_pscr;
      plan.head_group = head_group;
      plan.pinv = d.d_pscr + (size_t)head_group * max_p;
      plan.pinv_ld = (int)max_t;
    }
    auto forward = [&]() {
      return forward_mb(m, d, d_ids + mb.t0, d.d_meta + mb.cu_off, mb.s1 - mb.s0, mb.t1 - mb.t0,
                        mb.sum_l2, plan, out_dim, d_out + (size_t)mb.s0 * dim, st, cancel, err,
                        errlen);
    };
    // A small one-micro-batch call replays the graph of an earlier call with
    // the same launches (this call's ids and metadata were uploaded above, to
    // the same addresses). Its cancellation is checked at entry and before
    // the micro-batch; the layer checkpoints pass at capture. Profiling and
    // the debug cancellation counter keep the direct launches.
    const bool graph = allow_graph && mbs.size() == 1 && mb.t1 - mb.t0 <= kGraphMaxTokens &&
                       !d.prof_on && t_cancel_after < 0;
    if (!graph) {
      if ((rc = forward())) return rc;
    } else {
      const std::vector<long long> key = {
          mb.t1 - mb.t0, mb.s1 - mb.s0, out_dim, mb.ntiles, mb.nwin, mb.nseg,
          (long long)mb.cu_off, (long long)mb.tile_off, (long long)mb.cls_off,
          (long long)mb.win_off, (long long)mb.seg_off, (long long)mb.poff_off,
          (long long)mb.pcls_off, (long long)mb.ptot, (long long)mb.ptot_cls, head_group,
          (long long)max_p, (long long)max_t, (long long)(intptr_t)d_ids,
          (long long)(intptr_t)d_out, (long long)(intptr_t)d.d_meta,
          (long long)(intptr_t)d.d_pscr, (long long)(intptr_t)d.ws.base,
          (long long)d.ws.tokens, (long long)(intptr_t)st};
      auto it = d.graphs.find(key);
      if (it == d.graphs.end()) {
        // Capture this call's launches (they run when the graph is launched
        // below); any capture failure falls back to direct launches.
        const long long l0 = d.launches.load();
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed) != cudaSuccess) {
          (void)cudaGetLastError();
          if ((rc = forward())) return rc;
        } else {
          // The float path's kernels (and the default attention) wait for
          // their predecessor before touching global memory, so inside its
          // graph each may start while the previous one finishes.
          d.pdl = !m.q8 && m.attn_kind == kAttnHeads;
          rc = forward();
          d.pdl = false;
          const cudaError_t ce = cudaStreamEndCapture(st, &g);
          cudaGraphExec_t ex = nullptr;
          const bool ok = ce == cudaSuccess && g && cudaGraphInstantiate(&ex, g, 0) == cudaSuccess;
          if (g) cudaGraphDestroy(g);
          if (rc) {
            if (ex) cudaGraphExecDestroy(ex);
            return rc;
          }
          if (!ok) {
            (void)cudaGetLastError();
            if ((rc = forward())) return rc;
          } else {
            if (d.graphs.size() >= kGraphCacheSize) {  // drop the least recently used
              auto lru = d.graphs.begin();
              for (auto j = d.graphs.begin(); j != d.graphs.end(); ++j)
                if (j->second.used < lru->second.used) lru = j;
              cudaGraphExecDestroy(lru->second.exec);
              d.graphs.erase(lru);
            }
            DevCtx::GraphEntry e;
            e.exec = ex;
            e.launches = d.launches.load() - l0;
            it = d.graphs.emplace(key, e).first;
            it->second.used = ++d.graph_clock;
            CU_TRY(cudaGraphLaunch(ex, st));
          }
        }
      } else {
        it->second.used = ++d.graph_clock;
        CU_TRY(cudaGraphLaunch(it->second.exec, st));
        d.launches.fetch_add(it->second.launches, std::memory_order_relaxed);
      }
    }
    if (after_mb && (rc = after_mb((int)i, mb.s0, mb.s1))) return rc;
  }
  return FUTON_OK;
}

// The device error word of the calls so far: read here (a blocking copy), or
// taken from *copied, an asynchronous copy of it the caller queued after its
// kernels and has synchronised.
int read_device_error(DevCtx& d, char* err, size_t errlen, const int* copied = nullptr) {
  int code = 0;
  if (copied) {
    code = *copied;
  } else {
    CU_TRY(cudaMemcpy(&code, d.err_word, sizeof(int), cudaMemcpyDeviceToHost));
  }
  d.d2h_bytes.fetch_add((long long)sizeof(int), std::memory_order_relaxed);
  if (code != 0) {
    // Cleared on the device's stream (ordered with the next call's kernels).
    CU_TRY(cudaMemsetAsync(d.err_word, 0, sizeof(int), d.stream));
    CU_TRY(cudaStreamSynchronize(d.stream));
    return set_err(err, errlen, code == kDevBadInput ? FUTON_EINVAL : FUTON_EDEVICE,
                   code == kDevBadInput ? "native: token id outside vocab (device-side check)"
                                        : "native: device-side error %d (a bounded pipeline wait expired)",
                   code);
  }
  return FUTON_OK;
}

// Host-buffer encode on one device (blocking).
int encode_host(futon_model* m, DevCtx& d, const int32_t* ids, const int32_t* cu, int nseq,
                int out_dim, float* out, volatile const int* cancel, char* err, size_t errlen) {
  std::lock_guard<std::mutex> lock(d.mu);
  CU_TRY(cudaSetDevice(d.device));
  if (nseq == 0) return FUTON_OK;
  const size_t T = (size_t)cu[nseq];
  const int dim = out_dim ? out_dim : m->cfg.hidden_size;
  int rc;
  if ((rc = ensure_host(&d.h_ids, &d.h_ids_cap, T, err, errlen))) return rc;
  if ((rc = ensure_dev(&d.d_ids, &d.d_ids_cap, T, err, errlen))) return rc;
  if ((rc = ensure_host(&d.h_out, &d.h_out_cap, (size_t)nseq * dim, err, errlen))) return rc;
  if ((rc = ensure_dev(&d.d_out, &d.d_out_cap, (size_t)nseq * dim, err, errlen))) return rc;
  // The ids of the first micro-batch (at most kTokenBudget tokens: all of a
  // small call) go up before planning; the rest micro-batch by micro-batch,
  // just before each forward (the host copies micro-batch i + 1's while the
  // GPU runs i). `sent`: tokens [0, sent) are on their way.
  size_t sent = 0;
  auto send_ids = [&](size_t t1) -> int {
    if (t1 <= sent) return FUTON_OK;
    const size_t n = t1 - sent;
    memcpy(d.h_ids + sent, ids + sent, n * sizeof(int));
    CU_TRY(cudaMemcpyAsync(d.d_ids + sent, d.h_ids + sent, n * sizeof(int),
                           cudaMemcpyHostToDevice, d.stream));
    d.h2d_bytes.fetch_add((long long)(n * sizeof(int)), std::memory_order_relaxed);
    sent = t1;
    return FUTON_OK;
  };
  if ((rc = send_ids(std::min(T, (size_t)kTokenBudget)))) return rc;
  auto before_mb = [&](int, int, int t1) -> int { return send_ids((size_t)t1); };
  // Each micro-batch's vectors go to pinned memory as soon as it is done
  // (event per micro-batch); this thread copies them out to `out` while the
  // GPU works on the next micro-batches.
  struct Done { int s0, s1; };
  std::vector<Done> done;
  auto after_mb = [&](int i, int s0, int s1) -> int {
    while ((int)d.out_evts.size() <= i) {
      cudaEvent_t e = nullptr;
      CU_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      d.out_evts.push_back(e);
    }
    CU_TRY(cudaMemcpyAsync(d.h_out + (size_t)s0 * dim, d.d_out + (size_t)s0 * dim,
                           (size_t)(s1 - s0) * dim * sizeof(float), cudaMemcpyDeviceToHost,
                           d.stream));
    d.d2h_bytes.fetch_add((long long)((size_t)(s1 - s0) * dim * sizeof(float)),
                          std::memory_order_relaxed);
    CU_TRY(cudaEventRecord(d.out_evts[i], d.stream));
    done.push_back(Done{s0, s1});
    return FUTON_OK;
  };
  rc = run_call(*m, d, d.d_ids, cu, nseq, out_dim, d.d_out, d.stream, cancel, err, errlen, after_mb,
                before_mb, /*allow_graph=*/true);
  if (rc) {
    cudaStreamSynchronize(d.stream);  // leave nothing in flight
    return rc;
  }
  // The error word comes back behind the last vectors (no second round trip).
  if ((rc = ensure_host(&d.h_err, &d.h_err_cap, 1, err, errlen))) return rc;
  CU_TRY(cudaMemcpyAsync(d.h_err, d.err_word, sizeof(int), cudaMemcpyDeviceToHost, d.stream));
  for (size_t i = 0; i < done.size(); ++i) {
    CU_TRY(cudaEventSynchronize(d.out_evts[i]));
    const size_t off = (size_t)done[i].s0 * dim, n = (size_t)(done[i].s1 - done[i].s0) * dim;
    memcpy(out + off, d.h_out + off, n * sizeof(float));
  }
  CU_TRY(cudaStreamSynchronize(d.stream));
  return read_device_error(d, err, errlen, d.h_err);
}

// ---- kernel-seam context (per CUDA device) ------------------------------
struct SeamCtx {
  std::mutex mu;
  void* scratch = nullptr;
  size_t cap = 0;
  int* err_word = nullptr;
  int num_sms = 148;
  bool init = false;
};
SeamCtx g_seam[64];

// Takes the device's seam lock (handed to the caller in *lk, held until the
// call returns: the scratch, its capacity and the error word are shared by
// every seam call on the device), then initialises the context and grows
// the scratch to `bytes`.
int seam_begin(int dev, size_t bytes, SeamCtx** out, std::unique_lock<std::mutex>* lk, char* err,
               size_t errlen) {
  if (dev < 0 || dev >= 64) return set_err(err, errlen, FUTON_EINVAL, "native: bad device %d", dev);
  SeamCtx& s = g_seam[dev];
  std::unique_lock<std::mutex> held(s.mu);
  CU_TRY(cudaSetDevice(dev));
  if (!s.init) {
    CU_TRY(cudaMalloc(&s.err_word, sizeof(int)));
    CU_TRY(cudaMemset(s.err_word, 0, sizeof(int)));
    CU_TRY(cudaDeviceSynchronize());  // zero before kernels on any stream read it
    CU_TRY(cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev));
    s.init = true;
  }
  if (s.cap < bytes) {
    CU_TRY(cudaDeviceSynchronize());
    if (s.scratch) cudaFree(s.scratch);
    s.scratch = nullptr;
    s.cap = 0;
    CU_TRY(cudaMalloc(&s.scratch, bytes));
    s.cap = bytes;
  }
  *out = &s;
  *lk = std::move(held);
  return FUTON_OK;
}

int seam_finish(SeamCtx& s, cudaStream_t st, char* err, size_t errlen) {
  CU_TRY(cudaStreamSynchronize(st));
  int code = 0;
  CU_TRY(cudaMemcpy(&code, s.err_word, sizeof(int), cudaMemcpyDeviceToHost));
  if (code) {
    CU_TRY(cudaMemsetAsync(s.err_word, 0, sizeof(int), st));
    CU_TRY(cudaStreamSynchronize(st));
    return set_err(err, errlen, FUTON_EDEVICE, "native: device-side error %d", code);
  }
  return FUTON_OK;
}

// The kernel seam's GEMM launch (f32 output, bias, optional int8 rescale),
// shared by the allocating seam calls and the no-allocation Q8 entry point:
// err_word is the device error word the kernel's bounded waits report into.
int seam_gemm(int* err_word, int num_sms, const void* A, bool s8, const float* a_scale, int m,
              const void* W, const float* w_scale, int n, int k, const float* bias, float* dst,
              cudaStream_t st, char* err, size_t errlen) {
  CUtensorMap ta, tw;
  const int bn = pick_bn(n);
  const Elem el = s8 ? kElemS8 : kElemBf16;
  if (!make_operand_map(&ta, A, el, (uint64_t)m, (uint64_t)k, 128) ||
      !make_operand_map(&tw, W, el, (uint64_t)n, (uint64_t)k, (uint32_t)bn))
    return set_err(err, errlen, FUTON_ECUDA, "native: cuTensorMapEncodeTiled failed");
  GemmLaunch g;
  g.ta = &ta;
  g.tw = &tw;
  g.to = nullptr;
  g.tr = nullptr;
  g.M = m;
  g.N = n;
  g.K = k;
  g.bn = bn;
  g.epi = kEpiStore;
  g.out_f32 = true;
  g.f16 = false;
  g.pair = false;
  g.pdl = false;
  g.ep.out = dst;
  g.ep.ldo = n;
  g.ep.bias = bias;
  g.ep.resid = nullptr;
  g.ep.ldr = 0;
  g.ep.resid_kind = kResidF32;
  g.ep.a_scale = a_scale;
  g.ep.w_scale = w_scale;
  g.ep.ln_w = nullptr;
  g.ep.ln_b = nullptr;
  g.ep.eps = 0.f;
  g.ep.out_f32 = nullptr;
  g.ep.rope_cos = nullptr;
  g.ep.rope_sin = nullptr;
  g.ep.rope_hd = 0;
  g.ep.rope_cols = 0;
  g.ep.cu = nullptr;
  g.ep.nseq = 0;
  g.ep.f16_from = 1 << 30;
  g.err = err_word;
  g.num_sms = num_sms;
  g.stream = st;
  cudaError_t e = s8 ? launch_gemm_s8(g) : launch_gemm_bf16(g);
  if (e != cudaSuccess)
    return set_err(err, errlen, FUTON_ECUDA, "native: gemm launch: %s", cudaGetErrorString(e));
  return FUTON_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int futon_cuda_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

static int futon_cuda_model_create_impl(const futon_cfg* cfg, const futon_tensor* tensors, int ntensors,
                            const int* devices, int ndev, int q8, futon_model** out, char* err,
                            size_t errlen) {
  if (!cfg || !out || (ntensors > 0 && !tensors))
    return set_err(err, errlen, FUTON_EINVAL, "native: null argument");
  *out = nullptr;
  const futon_cfg& c = *cfg;
  const int h = c.hidden_size, I = c.intermediate_size, H = c.num_heads;
  if (h <= 0 || c.num_layers <= 0 || H <= 0 || I <= 0 || c.vocab_size <= 0 || c.max_seq_len <= 2)
    return set_err(err, errlen, FUTON_EINVAL, "native: non-positive architecture dimension");
  if (h % H != 0)
    return set_err(err, errlen, FUTON_EINVAL, "native: hidden_size %d not divisible by num_heads %d", h, H);
  const int hd = h / H;
  if (h % 8 || I % 8 || h > 1024)
    return set_err(err, errlen, FUTON_EINVAL,
                   "native: hidden_size and intermediate_size must be multiples of 8 (hidden ≤ 1024)");
  if (q8 && (h % 16 || I % 16))
    return set_err(err, errlen, FUTON_EINVAL, "native: the int8 path needs K multiples of 16");
  if (hd != 8 && hd != 16 && hd != 32 && hd != 64)
    return set_err(err, errlen, FUTON_EINVAL, "native: unsupported head_dim %d", hd);
  const bool rope = c.position_encoding == FUTON_POS_ROPE, swiglu = c.activation == FUTON_ACT_SWIGLU;
  if (rope && !(c.rope_theta > 0))
    return set_err(err, errlen, FUTON_EINVAL, "native: rope position encoding requires rope_theta > 0");
  int half = 0;
  if (swiglu) {
    half = (I % 128 == 0) ? 128 : (I % 64 == 0) ? 64 : (I % 32 == 0) ? 32 : 0;
    if (!half)
      return set_err(err, errlen, FUTON_EINVAL, "native: swiglu needs intermediate_size %% 32 == 0");
  }
  if (!devices || ndev <= 0) return set_err(err, errlen, FUTON_EINVAL, "native: no devices");
  int visible = futon_cuda_device_count();
  for (int i = 0; i < ndev; ++i)
    if (devices[i] < 0 || devices[i] >= visible)
      return set_err(err, errlen, FUTON_EINVAL, "native: device %d not visible (%d devices)",
                     devices[i], visible);

  // ---- tensor set (newModel, model.go:134-263) ----
  TensorSet ts;
  for (int i = 0; i < ntensors; ++i) {
    const futon_tensor& t = tensors[i];
    if (!t.name || !t.data)
      return set_err(err, errlen, FUTON_EINVAL, "native: tensor %d has no name or data", i);
    if (t.dtype != FUTON_DTYPE_F32 && t.dtype != FUTON_DTYPE_F16)
      return set_err(err, errlen, FUTON_EINVAL, "native: tensor %s has unsupported dtype", t.name);
    if (t.ndim < 1 || t.ndim > 4)
      return set_err(err, errlen, FUTON_EINVAL, "native: tensor %s has rank %d", t.name, t.ndim);
    HostTensor ht;
    ht.t = &t;
    if (ts.byname.count(t.name))
      return set_err(err, errlen, FUTON_EINVAL, "native: duplicate tensor %s", t.name);
    ts.byname.emplace(t.name, std::move(ht));
  }
  int rc;
  const float *word, *pos = nullptr, *type = nullptr, *embw, *embb;
  if ((rc = need(ts, "embeddings.word", {c.vocab_size, h}, false, &word, err, errlen))) return rc;
  if (!rope && (rc = need(ts, "embeddings.position", {c.max_seq_len, h}, false, &pos, err, errlen))) return rc;
  if (c.type_vocab_size > 0 &&
      (rc = need(ts, "embeddings.token_type", {c.type_vocab_size, h}, false, &type, err, errlen)))
    return rc;
  if ((rc = need(ts, "embeddings.norm.weight", {h}, false, &embw, err, errlen))) return rc;
  if ((rc = need(ts, "embeddings.norm.bias", {h}, false, &embb, err, errlen))) return rc;
  struct LW {
    HostMat qkvw, outw, fc1w, gatew, fc2w;
    const float *qkvb, *outb, *n1w, *n1b, *fc1b, *gateb, *fc2b, *n2w, *n2b;
  };
  std::vector<LW> lw(c.num_layers);
  for (int i = 0; i < c.num_layers; ++i) {
    auto p = [&](const char* s) { return "layers." + std::to_string(i) + "." + s; };
    LW& l = lw[i];
    l.gateb = nullptr;
    if ((rc = need_mat(ts, p("attn.qkv.weight"), {3 * h, h}, &l.qkvw, err, errlen))) return rc;
    if ((rc = need(ts, p("attn.qkv.bias"), {3 * h}, true, &l.qkvb, err, errlen))) return rc;
    if ((rc = need_mat(ts, p("attn.out.weight"), {h, h}, &l.outw, err, errlen))) return rc;
    if ((rc = need(ts, p("attn.out.bias"), {h}, true, &l.outb, err, errlen))) return rc;
    if ((rc = need(ts, p("norm1.weight"), {h}, false, &l.n1w, err, errlen))) return rc;
    if ((rc = need(ts, p("norm1.bias"), {h}, false, &l.n1b, err, errlen))) return rc;
    if ((rc = need_mat(ts, p("mlp.fc1.weight"), {I, h}, &l.fc1w, err, errlen))) return rc;
    if ((rc = need(ts, p("mlp.fc1.bias"), {I}, true, &l.fc1b, err, errlen))) return rc;
    if (swiglu) {
      if ((rc = need_mat(ts, p("mlp.gate.weight"), {I, h}, &l.gatew, err, errlen))) return rc;
      if ((rc = need(ts, p("mlp.gate.bias"), {I}, true, &l.gateb, err, errlen))) return rc;
    }
    if ((rc = need_mat(ts, p("mlp.fc2.weight"), {h, I}, &l.fc2w, err, errlen))) return rc;
    if ((rc = need(ts, p("mlp.fc2.bias"), {h}, true, &l.fc2b, err, errlen))) return rc;
    if ((rc = need(ts, p("norm2.weight"), {h}, false, &l.n2w, err, errlen))) return rc;
    if ((rc = need(ts, p("norm2.bias"), {h}, false, &l.n2b, err, errlen))) return rc;
  }
  for (auto& kv : ts.byname)
    if (!ts.used.count(kv.first))
      return set_err(err, errlen, FUTON_EINVAL,
                     "native: unexpected tensor %s (pack/config mismatch)", kv.first.c_str());

  auto model = std::make_unique<futon_model>();
  model->cfg = c;
  model->q8 = q8 ? 1 : 0;
  model->head_dim = hd;
  model->eff_max = effective_max(c);
  model->swiglu_half = half;
  model->fuse_ln = !q8 && h % ln_slice_cols(h) == 0 && h / ln_slice_cols(h) >= 2 &&
                   h / ln_slice_cols(h) <= kLnPeerSlots;
  read_attn_env(*model);

  // RoPE tables (precomputeRoPE, model.go:306-318): f64 angles, f32 storage.
  std::vector<float> rc_tab, rs_tab;
  if (rope) {
    const int ms = model->eff_max, hh = hd / 2;
    rc_tab.resize((size_t)ms * hh);
    rs_tab.resize((size_t)ms * hh);
    // cos and sin in loops of their own: one loop with both lets the
    // compiler fuse them into a sincos call, whose last bit may differ from
    // the separate calls the reference (and the test oracle) make.
    auto angle = [&](int t, int i) {
      const double freq = 1.0 / std::pow(c.rope_theta, (double)(2 * i) / (double)hd);
      return (double)t * freq;
    };
    for (int t = 0; t < ms; ++t)
      for (int i = 0; i < hh; ++i) rc_tab[(size_t)t * hh + i] = (float)std::cos(angle(t, i));
    for (int t = 0; t < ms; ++t)
      for (int i = 0; i < hh; ++i) rs_tab[(size_t)t * hh + i] = (float)std::sin(angle(t, i));
  }

  // One weight replica per device, uploaded by one host thread per device
  // (each GPU's copies run over its own link at the same time).
  const size_t max_mat = std::max<size_t>((size_t)3 * h * h, (size_t)2 * I * h);
  auto upload_device = [&](int dev, std::unique_ptr<DevCtx>* slot, char* e, size_t el) -> int {
    auto d = std::make_unique<DevCtx>();
    d->device = dev;
    char* err = e;
    size_t errlen = el;
    int rc;
    CU_TRY(cudaSetDevice(d->device));
    CU_TRY(cudaDeviceGetAttribute(&d->num_sms, cudaDevAttrMultiProcessorCount, d->device));
    d->gemm_pair = model->gemm_pair;
    CU_TRY(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking));
    CU_TRY(cudaEventCreateWithFlags(&d->meta_evt, cudaEventDisableTiming));
    CU_TRY(cudaEventRecord(d->meta_evt, d->stream));
    CU_TRY(cudaEventCreateWithFlags(&d->done_evt, cudaEventDisableTiming));
    CU_TRY(cudaEventRecord(d->done_evt, d->stream));
    if ((rc = dev_alloc(*d, &d->err_word, 1, err, errlen))) return rc;
    CU_TRY(cudaMemsetAsync(d->err_word, 0, sizeof(int), d->stream));
    if ((rc = upload_f32(*d, &d->word, word, (size_t)c.vocab_size * h, err, errlen))) return rc;
    if ((rc = upload_f32(*d, &d->pos, pos, pos ? (size_t)c.max_seq_len * h : 0, err, errlen))) return rc;
    if ((rc = upload_f32(*d, &d->type0, type, type ? (size_t)h : 0, err, errlen))) return rc;
    if ((rc = upload_f32(*d, &d->embw, embw, h, err, errlen))) return rc;
    if ((rc = upload_f32(*d, &d->embb, embb, h, err, errlen))) return rc;
    if (rope) {
      if ((rc = upload_f32(*d, &d->rcos, rc_tab.data(), rc_tab.size(), err, errlen))) return rc;
      if ((rc = upload_f32(*d, &d->rsin, rs_tab.data(), rs_tab.size(), err, errlen))) return rc;
    }
    void* staging = nullptr;
    CU_TRY(cudaMalloc(&staging, max_mat * 6));
    d->layers.resize(c.num_layers);
    const HostMat none;
    rc = FUTON_OK;
    for (int i = 0; i < c.num_layers && rc == FUTON_OK; ++i) {
      const LW& l = lw[i];
      LayerDev& L = d->layers[i];
      const bool fr = model->fuse_ln;
      if ((rc = upload_gemm(*d, L.qkv, l.qkvw, l.qkvb, none, nullptr, 3 * h, h, 0, q8, false, staging, err, errlen))) break;
      if ((rc = upload_gemm(*d, L.out, l.outw, l.outb, none, nullptr, h, h, 0, q8, fr, staging, err, errlen))) break;
      if (swiglu) rc = upload_gemm(*d, L.fc1, l.fc1w, l.fc1b, l.gatew, l.gateb, I, h, half, q8, false, staging, err, errlen);
      else rc = upload_gemm(*d, L.fc1, l.fc1w, l.fc1b, none, nullptr, I, h, 0, q8, false, staging, err, errlen);
      if (rc) break;
      if ((rc = upload_gemm(*d, L.fc2, l.fc2w, l.fc2b, none, nullptr, h, I, 0, q8, fr, staging, err, errlen))) break;
      if ((rc = upload_f32(*d, &L.n1w, l.n1w, h, err, errlen))) break;
      if ((rc = upload_f32(*d, &L.n1b, l.n1b, h, err, errlen))) break;
      if ((rc = upload_f32(*d, &L.n2w, l.n2w, h, err, errlen))) break;
      if ((rc = upload_f32(*d, &L.n2b, l.n2b, h, err, errlen))) break;
    }
    cudaFree(staging);
    if (rc) return rc;
    CU_TRY(cudaStreamSynchronize(d->stream));
    *slot = std::move(d);
    return FUTON_OK;
  };
  std::vector<std::unique_ptr<DevCtx>> devs(ndev);
  std::vector<int> rcs(ndev, FUTON_OK);
  std::vector<std::string> msgs(ndev);
  auto run_one = [&](int di) {
    char e[512] = {0};
    try {
      rcs[di] = upload_device(devices[di], &devs[di], e, sizeof e);
      msgs[di] = e;
    } catch (...) {
      rcs[di] = FUTON_ENOMEM;
      msgs[di] = "native: host exception while uploading a device replica";
    }
  };
  if (ndev == 1) {
    run_one(0);
  } else {
    run_on_threads(ndev, run_one);
  }
  for (int di = 0; di < ndev; ++di)
    if (rcs[di]) return set_err(err, errlen, rcs[di], "%s", msgs[di].c_str());
  for (auto& d : devs) model->devs.push_back(std::move(d));
  *out = model.release();
  return FUTON_OK;
}

int futon_cuda_model_create(const futon_cfg* cfg, const futon_tensor* tensors, int ntensors,
                            const int* devices, int ndev, int q8, futon_model** out, char* err,
                            size_t errlen) {
  try {
    return futon_cuda_model_create_impl(cfg, tensors, ntensors, devices, ndev, q8, out, err, errlen);
  }
  FUTON_CATCH(err, errlen)
}

void futon_cuda_model_destroy(futon_model* model) {
  if (!model) return;
  delete model;
}

static int futon_cuda_encode_impl(futon_model* model, int device, const int32_t* ids,
                      const int32_t* cu_seqlens, int nseq, int out_dim, float* out,
                      volatile const int* cancel, char* err, size_t errlen) {
  if (!model) return set_err(err, errlen, FUTON_EINVAL, "native: null model");
  if (device < 0 || device >= (int)model->devs.size())
    return set_err(err, errlen, FUTON_EINVAL, "native: device index %d out of range", device);
  if (nseq > 0 && (!ids || !cu_seqlens || !out))
    return set_err(err, errlen, FUTON_EINVAL, "native: null buffer");
  int rc;
  if ((rc = validate_input(*model, cu_seqlens, nseq, out_dim, err, errlen))) return rc;
  if ((rc = check_ids(*model, ids, cu_seqlens, nseq, err, errlen))) return rc;
  if (canceled(cancel)) return set_err(err, errlen, FUTON_ECANCELED, "native: context canceled");
  return encode_host(model, *model->devs[device], ids, cu_seqlens, nseq, out_dim, out, cancel, err,
                     errlen);
}

int futon_cuda_encode(futon_model* model, int device, const int32_t* ids,
                      const int32_t* cu_seqlens, int nseq, int out_dim, float* out,
                      volatile const int* cancel, char* err, size_t errlen) {
  try {
    return futon_cuda_encode_impl(model, device, ids, cu_seqlens, nseq, out_dim, out, cancel, err, errlen);
  }
  FUTON_CATCH(err, errlen)
}

static int futon_cuda_encode_batch_impl(futon_model* model, const int32_t* ids, const int32_t* cu_seqlens,
                            int nseq, int out_dim, float* out, volatile const int* cancel,
                            char* err, size_t errlen) {
  if (!model) return set_err(err, errlen, FUTON_EINVAL, "native: null model");
  if (nseq > 0 && (!ids || !cu_seqlens || !out))
    return set_err(err, errlen, FUTON_EINVAL, "native: null buffer");
  int rc;
  if ((rc = validate_input(*model, cu_seqlens, nseq, out_dim, err, errlen))) return rc;
  if ((rc = check_ids(*model, ids, cu_seqlens, nseq, err, errlen))) return rc;
  if (canceled(cancel)) return set_err(err, errlen, FUTON_ECANCELED, "native: context canceled");
  const int ndev = (int)model->devs.size();
  const int dim = out_dim ? out_dim : model->cfg.hidden_size;
  if (nseq == 0) return FUTON_OK;
  // Contiguous shards balanced by estimated cost: GEMM work ∝ L, attention ∝ L².
  const double h = model->cfg.hidden_size;
  std::vector<double> cost(nseq + 1, 0.0);
  for (int s = 0; s < nseq; ++s) {
    const double L = cu_seqlens[s + 1] - cu_seqlens[s];
    cost[s + 1] = cost[s] + L * (12.0 * h + 2.0 * L);
  }
  std::vector<int> cut(ndev + 1, nseq);
  cut[0] = 0;
  for (int k = 1; k < ndev; ++k) {
    const double target = cost[nseq] * k / ndev;
    cut[k] = (int)(std::lower_bound(cost.begin(), cost.end(), target) - cost.begin());
    cut[k] = std::max(cut[k - 1], std::min(cut[k], nseq));
  }
  std::vector<int> rcs(ndev, FUTON_OK);
  std::vector<std::string> msgs(ndev);
  run_on_threads(ndev, [&](int k) {
    const int s0 = cut[k], s1 = cut[k + 1];
    if (s1 <= s0) return;
    try {
      std::vector<int32_t> cu(s1 - s0 + 1);
      for (int s = s0; s <= s1; ++s) cu[s - s0] = cu_seqlens[s] - cu_seqlens[s0];
      char e[512] = {0};
      rcs[k] = encode_host(model, *model->devs[k], ids + cu_seqlens[s0], cu.data(), s1 - s0,
                           out_dim, out + (size_t)s0 * dim, cancel, e, sizeof e);
      msgs[k] = e;
    } catch (...) {
      rcs[k] = FUTON_ENOMEM;
      msgs[k] = "native: host exception in a device's shard";
    }
  });
  for (int k = 0; k < ndev; ++k)
    if (rcs[k] != FUTON_OK) return set_err(err, errlen, rcs[k], "%s", msgs[k].c_str());
  return FUTON_OK;
}

int futon_cuda_encode_batch(futon_model* model, const int32_t* ids, const int32_t* cu_seqlens,
                            int nseq, int out_dim, float* out, volatile const int* cancel,
                            char* err, size_t errlen) {
  try {
    return futon_cuda_encode_batch_impl(model, ids, cu_seqlens, nseq, out_dim, out, cancel, err, errlen);
  }
  FUTON_CATCH(err, errlen)
}

static int futon_cuda_encode_device_impl(futon_model* model, int device, const int32_t* d_ids,
                             const int32_t* cu_seqlens, int nseq, int out_dim, float* d_out,
                             void* stream, char* err, size_t errlen) {
  if (!model) return set_err(err, errlen, FUTON_EINVAL, "native: null model");
  if (device < 0 || device >= (int)model->devs.size())
    return set_err(err, errlen, FUTON_EINVAL, "native: device index %d out of range", device);
  if (nseq > 0 && (!d_ids || !d_out))
    return set_err(err, errlen, FUTON_EINVAL, "native: null buffer");
  int rc;
  if ((rc = validate_input(*model, cu_seqlens, nseq, out_dim, err, errlen))) return rc;
  DevCtx& d = *model->devs[device];
  std::lock_guard<std::mutex> lock(d.mu);
  CU_TRY(cudaSetDevice(d.device));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : d.stream;
  return run_call(*model, d, (const int*)d_ids, cu_seqlens, nseq, out_dim, d_out, st, nullptr, err,
                  errlen);
}

int futon_cuda_encode_device(futon_model* model, int device, const int32_t* d_ids,
                             const int32_t* cu_seqlens, int nseq, int out_dim, float* d_out,
                             void* stream, char* err, size_t errlen) {
  try {
    return futon_cuda_encode_device_impl(model, device, d_ids, cu_seqlens, nseq, out_dim, d_out, stream, err, errlen);
  }
  FUTON_CATCH(err, errlen)
}

static int futon_cuda_sync_impl(futon_model* model, int device, void* stream, char* err, size_t errlen) {
  if (!model) return set_err(err, errlen, FUTON_EINVAL, "native: null model");
  if (device < 0 || device >= (int)model->devs.size())
    return set_err(err, errlen, FUTON_EINVAL, "native: device index %d out of range", device);
  DevCtx& d = *model->devs[device];
  std::lock_guard<std::mutex> lock(d.mu);
  CU_TRY(cudaSetDevice(d.device));
  if (stream) CU_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  CU_TRY(cudaStreamSynchronize(d.stream));
  return read_device_error(d, err, errlen);
}

int futon_cuda_sync(futon_model* model, int device, void* stream, char* err, size_t errlen) {
  try {
    return futon_cuda_sync_impl(model, device, stream, err, errlen);
  }
  FUTON_CATCH(err, errlen)
}

long long futon_cuda_launch_count(futon_model* model, int device) {
  if (!model || device < 0 || device >= (int)model->devs.size()) return -1;
  return model->devs[device]->launches.load();
}

static int futon_cuda_io_bytes_impl(futon_model* model, int device, long long* h2d, long long* d2h, char* err,
                        size_t errlen) {
  if (!model || device < 0 || device >= (int)model->devs.size())
    return set_err(err, errlen, FUTON_EINVAL, "native: bad model or device index");
  if (h2d) *h2d = model->devs[device]->h2d_bytes.load();
  if (d2h) *d2h = model->devs[device]->d2h_bytes.load();
  return FUTON_OK;
}

int futon_cuda_io_bytes(futon_model* model, int device, long long* h2d, long long* d2h, char* err,
                        size_t errlen) {
  try {
    return futon_cuda_io_bytes_impl(model, device, h2d, d2h, err, errlen);
  }
  FUTON_CATCH(err, errlen)
}

static int futon_cuda_profile_impl(futon_model* model, int device, int enable, char* err, size_t errlen) {
  if (!model || device < 0 || device >= (int)model->devs.size())
    return set_err(err, errlen, FUTON_EINVAL, "native: bad model or device index");
  DevCtx& d = *model->devs[device];
  std::lock_guard<std::mutex> lock(d.mu);
  CU_TRY(cudaSetDevice(d.device));
  CU_TRY(cudaDeviceSynchronize());
  prof_collect(d);
  for (auto& g : d.prof_agg) g = DevCtx::ProfAgg();
  d.prof_on = enable != 0;
  return FUTON_OK;
}

int futon_cuda_profile(futon_model* model, int device, int enable, char* err, size_t errlen) {
  try {
    return futon_cuda_profile_impl(model, device, enable, err, errlen);
  }
  FUTON_CATCH(err, errlen)
}

static int futon_cuda_profile_read_impl(futon_model* model, int device, int stage, double* ms,
                            long long* launches, double* flops, double* bytes, char* err,
                            size_t errlen) {
  if (!model || device < 0 || device >= (int)model->devs.size())
    return set_err(err, errlen, FUTON_EINVAL, "native: bad model or device index");
  if (stage < 0 || stage >= kNumStages)
    return set_err(err, errlen, FUTON_EINVAL, "native: profiler stage %d out of range", stage);
  DevCtx& d = *model->devs[device];
  std::lock_guard<std::mutex> lock(d.mu);
  CU_TRY(cudaSetDevice(d.device));
  CU_TRY(cudaDeviceSynchronize());
  prof_collect(d);
  const auto& g = d.prof_agg[stage];
  if (ms) *ms = g.ms;
  if (launches) *launches = g.n;
  if (flops) *flops = g.flops;
  if (bytes) *bytes = g.bytes;
  return FUTON_OK;
}

int futon_cuda_profile_read(futon_model* model, int device, int stage, double* ms,
                            long long* launches, double* flops, double* bytes, char* err,
                            size_t errlen) {
  try {
    return futon_cuda_profile_read_impl(model, device, stage, ms, launches, flops, bytes, err, errlen);
  }
  FUTON_CATCH(err, errlen)
}

int futon_cuda_profile_stage_count(void) { return kNumStages; }

const char* futon_cuda_profile_stage_name(int stage) {
  return (stage >= 0 && stage < kNumStages) ? kStageNames[stage] : "";
}

static int futon_cuda_matmul_t_impl(int cuda_device, float* dst, const float* a, const float* b, int m, int n,
                        int k, const float* bias, void* stream, char* err, size_t errlen) {
  if (m < 0 || n <= 0 || k <= 0 || k % 8)
    return set_err(err, errlen, FUTON_EINVAL, "native: matmul shape m=%d n=%d k=%d (k %% 8 == 0)", m, n, k);
  if (m == 0) return FUTON_OK;
  if (!dst || !a || !b) return set_err(err, errlen, FUTON_EINVAL, "native: null buffer");
  const size_t abytes = align_up((size_t)m * k * 2, 256), bbytes = align_up((size_t)n * k * 2, 256);
  SeamCtx* s;
  int rc;
  std::unique_lock<std::mutex> lock;
  if ((rc = seam_begin(cuda_device, abytes + bbytes, &s, &lock, err, errlen))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  bf16* ab = (bf16*)s->scratch;
  bf16* bb = (bf16*)((uint8_t*)s->scratch + abytes);
  f32_to_bf16_kernel<<<1024, 256, 0, st>>>(a, (size_t)m * k, ab);
  f32_to_bf16_kernel<<<1024, 256, 0, st>>>(b, (size_t)n * k, bb);
  CU_TRY(cudaGetLastError());
  if ((rc = seam_gemm(s->err_word, s->num_sms, ab, false, nullptr, m, bb, nullptr, n, k, bias, dst,
                      st, err, errlen)))
    return rc;
  return seam_finish(*s, st, err, errlen);
}

int futon_cuda_matmul_t(int cuda_device, float* dst, const float* a, const float* b, int m, int n,
                        int k, const float* bias, void* stream, char* err, size_t errlen) {
  try {
    return futon_cuda_matmul_t_impl(cuda_device, dst, a, b, m, n, k, bias, stream, err, errlen);
  }
  FUTON_CATCH(err, errlen)
}

static int futon_cuda_matmul_t_q8_impl(int cuda_device, float* dst, const float* a, const int8_t* qb,
                           const float* scales, int m, int n, int k, const float* bias,
                           void* stream, char* err, size_t errlen) {
  if (m < 0 || n <= 0 || k <= 0 || k % 16)
    return set_err(err, errlen, FUTON_EINVAL, "native: q8 matmul shape m=%d n=%d k=%d (k %% 16 == 0)", m, n, k);
  if (m == 0) return FUTON_OK;
  if (!dst || !a || !qb || !scales) return set_err(err, errlen, FUTON_EINVAL, "native: null buffer");
  const size_t qbytes = align_up((size_t)m * k, 256), sbytes = align_up((size_t)m * 4, 256);
  SeamCtx* s;
  int rc;
  std::unique_lock<std::mutex> lock;
  if ((rc = seam_begin(cuda_device, qbytes + sbytes, &s, &lock, err, errlen))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int8_t* qa = (int8_t*)s->scratch;
  float* sa = (float*)((uint8_t*)s->scratch + qbytes);
  quant_rows_kernel<<<grid_rows(m, 8, s->num_sms), 256, 0, st>>>(a, m, k, qa, sa);
  CU_TRY(cudaGetLastError());
  if ((rc = seam_gemm(s->err_word, s->num_sms, qa, true, sa, m, qb, scales, n, k, bias, dst, st,
                      err, errlen)))
    return rc;
  return seam_finish(*s, st, err, errlen);
}

int futon_cuda_matmul_t_q8(int cuda_device, float* dst, const float* a, const int8_t* qb,
                           const float* scales, int m, int n, int k, const float* bias,
                           void* stream, char* err, size_t errlen) {
  try {
    return futon_cuda_matmul_t_q8_impl(cuda_device, dst, a, qb, scales, m, n, k, bias, stream, err, errlen);
  }
  FUTON_CATCH(err, errlen)
}

static int futon_cuda_quantize_rows_q8_impl(int cuda_device, int8_t* dst, float* scales, const float* src,
                                int rows, int k, void* stream, char* err, size_t errlen) {
  if (rows < 0 || k <= 0 || k % 4)
    return set_err(err, errlen, FUTON_EINVAL, "native: quantize shape rows=%d k=%d (k %% 4 == 0)", rows, k);
  if (rows == 0) return FUTON_OK;
  if (!dst || !scales || !src) return set_err(err, errlen, FUTON_EINVAL, "native: null buffer");
  SeamCtx* s;
  int rc;
  std::unique_lock<std::mutex> lock;
  if ((rc = seam_begin(cuda_device, 256, &s, &lock, err, errlen))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  quant_rows_kernel<<<grid_rows(rows, 8, s->num_sms), 256, 0, st>>>(src, rows, k, dst, scales);
  CU_TRY(cudaGetLastError());
  return seam_finish(*s, st, err, errlen);
}

int futon_cuda_quantize_rows_q8(int cuda_device, int8_t* dst, float* scales, const float* src,
                                int rows, int k, void* stream, char* err, size_t errlen) {
  try {
    return futon_cuda_quantize_rows_q8_impl(cuda_device, dst, scales, src, rows, k, stream, err, errlen);
  }
  FUTON_CATCH(err, errlen)
}

}  // extern "C"

// ===========================================================================
// Q8 GEMM without allocation
//
// For callers that may not allocate device memory once they are running: a
// serving loop whose HBM is already reserved by another allocator (a PyTorch
// caching allocator or an inference-server arena can hold all free memory),
// or a latency-critical path that cannot afford cudaMalloc/cudaFree
// (cudaFree synchronises the whole device). The quantised activations and
// their scales go to a fixed array in this library's device image instead of
// allocated scratch. The array (kNoAllocScratchBytes) is resident on every
// GPU that loads the library, until the process exits.
//
// The array is part of this file's device code, which the CUDA runtime loads
// onto a device lazily (CUDA_MODULE_LOADING=LAZY is the default): the first
// call on a device, or any earlier call into the library that launches one of
// this file's kernels there, loads it and so reserves the array and the code
// in device memory. A caller that hands the free HBM to another allocator
// therefore makes its first call before doing so; from then on the calls
// allocate nothing.
// ===========================================================================
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB
__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
__device__ __align__(256) int g_noalloc_err;

struct NoAllocDev {
  bool ready = false;
  uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch
  int* err = nullptr;          // device address of g_noalloc_err
  int num_sms = 148;
};
NoAllocDev g_noalloc[64];
std::mutex g_noalloc_mu;

// Resolves the device addresses of the static arrays on the current device
// (host code must not use the arrays' names as device pointers).
int noalloc_setup(int dev, NoAllocDev** out, char* err, size_t errlen) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDev& s = g_noalloc[dev];
  if (!s.ready) {
    void* p = nullptr;
    CU_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    s.scratch = static_cast<uint8_t*>(p);
    CU_TRY(cudaGetSymbolAddress(&p, g_noalloc_err));
    s.err = static_cast<int*>(p);
    CU_TRY(cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev));
    s.ready = true;
  }
  *out = &s;
  return FUTON_OK;
}

}  // namespace

extern "C" int futon_cuda_matmul_t_q8_noalloc(int cuda_device, float* dst, const float* a,
                                              const int8_t* qb, const float* scales, int m, int n,
                                              int k, const float* bias, void* stream, char* err,
                                              size_t errlen) {
  if (cuda_device < 0 || cuda_device >= 64)
    return set_err(err, errlen, FUTON_EINVAL, "native: bad device %d", cuda_device);
  if (m < 0 || n <= 0 || k <= 0 || k % 16)
    return set_err(err, errlen, FUTON_EINVAL,
                   "native: q8 matmul shape m=%d n=%d k=%d (k %% 16 == 0)", m, n, k);
  const size_t qbytes = align_up((size_t)m * k, 256), need = qbytes + (size_t)m * 4;
  if (need > kNoAllocScratchBytes)
    return set_err(err, errlen, FUTON_EINVAL,
                   "native: q8 no-alloc scratch needs %zu bytes for m=%d k=%d; the fixed "
                   "scratch holds %zu (m·k rounded up to 256, plus 4·m)", need, m, k, kNoAllocScratchBytes);
  if (m == 0) return FUTON_OK;
  if (!dst || !a || !qb || !scales) return set_err(err, errlen, FUTON_EINVAL, "native: null buffer");
  CU_TRY(cudaSetDevice(cuda_device));
  NoAllocDev* s;
  int rc;
  if ((rc = noalloc_setup(cuda_device, &s, err, errlen))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int8_t* qa = reinterpret_cast<int8_t*>(s->scratch);
  float* sa = reinterpret_cast<float*>(s->scratch + qbytes);
  CU_TRY(cudaMemsetAsync(s->err, 0, sizeof(int), st));
  quant_rows_kernel<<<grid_rows(m, 8, s->num_sms), 256, 0, st>>>(a, m, k, qa, sa);
  CU_TRY(cudaGetLastError());
  if ((rc = seam_gemm(s->err, s->num_sms, qa, true, sa, m, qb, scales, n, k, bias, dst, st, err,
                      errlen)))
    return rc;
  CU_TRY(cudaStreamSynchronize(st));
  int code = 0;
  CU_TRY(cudaMemcpy(&code, s->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (code) return set_err(err, errlen, FUTON_EDEVICE, "native: device-side error %d", code);
  return FUTON_OK;
}

// ---- failure-detection self-test -------------------------------------------
namespace {
__global__ void selftest_wait_kernel(int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  // Phase 0 never completes: nothing arrives on the barrier.
  if (threadIdx.x == 0) mbar_wait_bounded(smem_u32(&bar), 0u, err, kDevTimeoutSelfTest, &abort_flag);
}
}  // namespace

extern "C" void futon_cuda_debug_cancel_after(long long polls) {
  t_cancel_after = polls < 0 ? -1 : polls;
}

static int futon_cuda_selftest_wait_timeout_impl(int cuda_device, char* err, size_t errlen) {
  SeamCtx* s = nullptr;
  int rc;
  std::unique_lock<std::mutex> lk;
  if ((rc = seam_begin(cuda_device, 0, &s, &lk, err, errlen))) return rc;
  CU_TRY(cudaMemset(s->err_word, 0, sizeof(int)));
  selftest_wait_kernel<<<1, 32>>>(s->err_word);
  CU_TRY(cudaGetLastError());
  CU_TRY(cudaDeviceSynchronize());
  int code = 0;
  CU_TRY(cudaMemcpy(&code, s->err_word, sizeof(int), cudaMemcpyDeviceToHost));
  CU_TRY(cudaMemset(s->err_word, 0, sizeof(int)));
  if (code != kDevTimeoutSelfTest)
    return set_err(err, errlen, FUTON_ECUDA,
                   "native: failure self-test: expected device code %d, read %d", kDevTimeoutSelfTest,
                   code);
  return set_err(err, errlen, FUTON_EDEVICE, "native: device wait timed out (self-test, code %d)",
                 code);
}

extern "C" int futon_cuda_selftest_wait_timeout(int cuda_device, char* err, size_t errlen) {
  try {
    return futon_cuda_selftest_wait_timeout_impl(cuda_device, err, errlen);
  }
  FUTON_CATCH(err, errlen)
}
