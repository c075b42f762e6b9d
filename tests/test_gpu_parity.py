"""GPU parity: libfuton_cuda (through its C ABI) against the CPU oracle, the
reference's golden vectors and the pinned torch restatement.

Gate for the f16 tensor-core path: per-vector cosine ≥ 0.9999 against the
reference algorithm and unit-norm outputs (|‖v‖ − 1| ≤ 1e-5).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN, GPU_COSINE_MIN, cosine, row_cosines
from futon_b200 import CancelFlag, CanceledError, FutonError, Model, synth
from futon_b200.pack import load_pack
from oracle.oracle import GEMM_AVX2, GEMM_GO, OracleModel, has_avx2

pytestmark = pytest.mark.gpu
NORM_TOL = 1e-5
_models = {}


def oracle_mode():
    return GEMM_AVX2 if has_avx2() else GEMM_GO


def synth_model(arch: str, q8: bool = False):
    key = (arch, q8)
    if key not in _models:
        cfg = synth.arch(arch)
        w = synth.make_weights(cfg)
        _models[key] = (cfg, w, Model(cfg, w, devices=[0], q8=q8))
    return _models[key]


def assert_parity(got, want, label, cos_min=GPU_COSINE_MIN):
    cs = row_cosines(got, want)
    norms = np.linalg.norm(got, axis=1)
    print(f"[parity] {label}: n={len(cs)} min cos {cs.min():.7f} mean {cs.mean():.7f} "
          f"max |norm-1| {np.abs(norms - 1).max():.1e}")
    assert cs.min() >= cos_min, f"{label}: min cosine {cs.min():.7f} < {cos_min} (mean {cs.mean():.7f})"
    assert np.abs(norms - 1).max() <= NORM_TOL, f"{label}: norm off by {np.abs(norms - 1).max():.2e}"
    return cs


# ---------------------------------------------------------------------------
# Reference golden vectors (native/testdata/toy/expected.json)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("pack", ["toy-absolute-gelu", "toy-rope-swiglu"])
def test_toy_golden(gpu, toy_expected, pack):
    p = load_pack(GOLDEN / pack)
    m = Model(p.cfg, p.tensors, devices=[0], q8=False)
    pexp = toy_expected["packs"][pack]
    worst = 1.0
    for c in pexp["forward_cases"]:
        got = m.encode_tokens(c["ids"])
        want = np.asarray(c["vector"], np.float32)
        worst = min(worst, cosine(got, want))
        assert cosine(got, want) >= GPU_COSINE_MIN, (pack, len(c["ids"]), cosine(got, want))
        assert np.abs(got - want).max() <= 5e-3
    for c in pexp.get("matryoshka_cases", []):
        got = m.encode_tokens(c["ids"], c["dim"])
        assert got.shape == (c["dim"],)
        assert cosine(got, np.asarray(c["vector"], np.float32)) >= GPU_COSINE_MIN
    for c in pexp.get("text_cases", []):
        got = m.encode_tokens(c["ids"])
        assert cosine(got, np.asarray(c["vector"], np.float32)) >= GPU_COSINE_MIN
    m.close()


def test_toy_golden_packed(gpu, toy_expected):
    """All forward cases of a pack in ONE packed call match the goldens."""
    for pack in ("toy-absolute-gelu", "toy-rope-swiglu"):
        p = load_pack(GOLDEN / pack)
        m = Model(p.cfg, p.tensors, devices=[0])
        cases = toy_expected["packs"][pack]["forward_cases"]
        from futon_b200 import pack_ids
        ids, cu = pack_ids([c["ids"] for c in cases])
        got = m.encode_packed(ids, cu)
        want = np.stack([np.asarray(c["vector"], np.float32) for c in cases])
        assert_parity(got, want, pack)
        m.close()


# ---------------------------------------------------------------------------
# Benchmark configurations vs the oracle
# ---------------------------------------------------------------------------
def test_c0_full_vs_oracle(gpu):
    cfg, w, m = synth_model("bge")
    ids, cu = synth.make_inputs("c0")
    got = m.encode_packed(ids, cu)
    want = OracleModel(cfg, w, gemm=oracle_mode()).encode_batch(ids, cu)
    cs = assert_parity(got, want, "c0")
    print(f"c0 min cos {cs.min():.7f} mean {cs.mean():.7f}")


@pytest.mark.parametrize("arch", ["bge", "nomic"])
def test_f16_pack_vs_oracle(gpu, arch):
    """Shipped packs store F16 tensors (safetensors.go:266-289; the reference
    expands them to f32 for MatMulTF16, kernel.go:38-42). The library takes
    them as F16 over the ABI and multiplies them as they are (f16 operands,
    f32 accumulation: no re-rounding of any weight); the oracle runs on
    their exact f32 expansion. Gate 0.99999, ten times tighter than the
    north-star 0.9999: weights rounded to bf16 on upload stay near 0.99996."""
    cfg = synth.arch(arch)
    cfg.num_layers = 3
    w16 = {k: v.astype(np.float16) for k, v in synth.make_weights(cfg).items()}
    m = Model(cfg, w16, devices=[0])
    ids, cu = synth.make_inputs("c0" if arch == "bge" else "c2", nseq=12, vocab=cfg.vocab_size)
    got = m.encode_packed(ids, cu)
    m.close()
    w32 = {k: v.astype(np.float32) for k, v in w16.items()}
    want = OracleModel(cfg, w32, gemm=oracle_mode()).encode_batch(ids, cu)
    assert_parity(got, want, f"f16 pack {arch}", cos_min=0.99999)


@pytest.mark.parametrize("heads", [3, 6])
def test_head_dim32_head_counts_vs_oracle(gpu, heads):
    """head_dim 32 with an odd head count (one head per attention step) and
    an even one (two heads per step), at widths the fused LayerNorm slices do
    not divide (standalone LayerNorm kernel), sequences up to 128 tokens (two
    key tiles)."""
    cfg = synth.arch("bge")
    cfg.hidden_size, cfg.num_heads, cfg.intermediate_size, cfg.num_layers = 32 * heads, heads, 128 * heads, 2
    w = synth.make_weights(cfg)
    m = Model(cfg, w, devices=[0])
    ids, cu = synth.make_inputs("c0", nseq=16, vocab=cfg.vocab_size)
    got = m.encode_packed(ids, cu)
    m.close()
    want = OracleModel(cfg, w, gemm=oracle_mode()).encode_batch(ids, cu)
    assert_parity(got, want, f"hd32 × {heads} heads")


def test_c1_full_vs_oracle(gpu):
    """c1 at full size: all 256 MiniLM-6 sequences of 128 tokens (mean
    pooling) against the oracle on every host core."""
    cfg, w, m = synth_model("minilm6")
    ids, cu = synth.make_inputs("c1")
    assert len(cu) - 1 == 256 and ids.size == 256 * 128
    got = m.encode_packed(ids, cu)
    want = OracleModel(cfg, w, gemm=oracle_mode()).encode_batch(ids, cu)
    assert_parity(got, want, "c1-full")


@pytest.mark.parametrize("dim", [768, 256, 64])
def test_c2_full_vs_oracle(gpu, dim):
    """c2 at full size: all 64 nomic-shaped sequences (lengths U[64, 512],
    RoPE, SwiGLU, mean pooling) at each matryoshka width."""
    cfg, w, m = synth_model("nomic")
    ids, cu = synth.make_inputs("c2")
    assert len(cu) - 1 == 64
    got = m.encode_packed(ids, cu, out_dim=dim)
    assert got.shape == (64, dim)
    want = OracleModel(cfg, w, gemm=oracle_mode()).encode_batch(ids, cu, out_dim=dim)
    assert_parity(got, want, f"c2-full/{dim}")


# Q8 path gates. The reference's Q8 forward quantises every layer's
# activations per row (48 times for 12 layers), so float32-rounding-level
# differences before a quantisation move whole int8 steps: 1e-7 relative
# noise on the attention output alone moves the vector to cos ≈ 0.9999. The
# device int8 path therefore repeats the reference's float32 operation order
# wherever a quantisation follows (attention in the avx2Kernel order,
# layerNormRows' sequential f64 statistics, the exact GELU/SiLU), and its
# vectors come out bit-identical to the oracle's Q8 forward in the
# avx2Kernel order. Gates: cos ≥ 0.99999 against that forward (the count of
# bit-identical vectors is printed) and the reference's own Q8 acceptance
# rule, cos ≥ 0.999 against the float path (native/quant.go:27-29).
Q8_COSINE_MIN = 0.99999
Q8_VS_FLOAT_MIN = 0.999


def _q8_oracle_or_skip():
    if not has_avx2():
        pytest.skip("the int8 path follows the reference's avx2Kernel order: needs an AVX2 host")
    return GEMM_AVX2


@pytest.mark.parametrize("q8", [False, True])
def test_c3_short_vs_oracle(gpu, q8):
    """arctic shape (RoPE, SwiGLU, CLS) at L=256 against the oracle, both
    the f32-weight path and the Q8 path (oracle requantises like model.go)."""
    gemm = _q8_oracle_or_skip() if q8 else oracle_mode()
    cfg, w, m = synth_model("arctic", q8=q8)
    rng = np.random.default_rng(5)
    lens = [256, 200]
    seqs = [np.concatenate([[101], rng.integers(1000, cfg.vocab_size, L - 2), [102]]) for L in lens]
    from futon_b200 import pack_ids
    ids, cu = pack_ids(seqs)
    got = m.encode_packed(ids, cu)
    want = OracleModel(cfg, w, q8=q8, gemm=gemm).encode_batch(ids, cu)
    assert_parity(got, want, f"c3 q8={q8}", Q8_COSINE_MIN if q8 else GPU_COSINE_MIN)
    if q8:
        flt = OracleModel(cfg, w, q8=False, gemm=oracle_mode()).encode_batch(ids, cu)
        assert_parity(got, flt, "c3 q8 vs float", Q8_VS_FLOAT_MIN)


@pytest.mark.parametrize("arch,inputs,nseq,layers", [
    ("bge", "c0", 16, None),  # absolute positions, GELU, CLS, head_dim 32
    ("nomic", "c2", 4, 2),    # mean pooling: every layer attends over all rows
    ("minilm6", "c1", 8, None),
])
def test_q8_bit_identical_to_oracle(gpu, arch, inputs, nseq, layers):
    """The int8 forward on every architecture: bit-identical vectors to the
    oracle's Q8 forward in the avx2Kernel order."""
    gemm = _q8_oracle_or_skip()
    cfg = synth.arch(arch)
    if layers:
        cfg.num_layers = layers
    w = synth.make_weights(cfg)
    m = Model(cfg, w, devices=[0], q8=True)
    ids, cu = synth.make_inputs(inputs, nseq=nseq, vocab=cfg.vocab_size)
    got = m.encode_packed(ids, cu)
    m.close()
    want = OracleModel(cfg, w, q8=True, gemm=gemm).encode_batch(ids, cu)
    same = int(np.sum(np.all(got == want, axis=1)))
    print(f"[q8] {arch}: {same}/{len(got)} vectors bit-identical")
    assert_parity(got, want, f"q8 {arch}", Q8_COSINE_MIN)
    assert same == len(got), f"{arch}: {len(got) - same} int8-path vectors differ from the oracle"


def test_q8_f16_pack_bit_identical(gpu):
    """An F16 pack on the int8 path: the weights are widened to f32 on the
    device and quantised per row there (quantizeRowQ8 of the exact f32
    expansion), so the vectors equal the oracle's Q8 forward bit for bit."""
    gemm = _q8_oracle_or_skip()
    cfg = synth.arch("nomic")
    cfg.num_layers = 2
    w16 = {k: v.astype(np.float16) for k, v in synth.make_weights(cfg).items()}
    m = Model(cfg, w16, devices=[0], q8=True)
    ids, cu = synth.make_inputs("c2", nseq=4, vocab=cfg.vocab_size)
    got = m.encode_packed(ids, cu)
    m.close()
    w32 = {k: v.astype(np.float32) for k, v in w16.items()}
    want = OracleModel(cfg, w32, q8=True, gemm=gemm).encode_batch(ids, cu)
    assert np.array_equal(got, want)


def test_c4_subset_vs_oracle(gpu):
    cfg, w, m = synth_model("bge")
    ids, cu = synth.make_inputs("c4", nseq=96)
    got = m.encode_packed(ids, cu)
    want = OracleModel(cfg, w, gemm=oracle_mode()).encode_batch(ids, cu)
    assert_parity(got, want, "c4-subset")


# ---------------------------------------------------------------------------
# Full-size: c3 at L=2048 vs the pinned torch restatement (fp32 on the GPU)
# ---------------------------------------------------------------------------
def test_c3_full_vs_torch(gpu):
    """c3 f32-weight path at full size (16 × 2048) against the oracle-pinned
    torch restatement on the GPU (the scalar oracle would take minutes)."""
    import torch
    from torch_ref import TorchRef
    torch.backends.cuda.matmul.allow_tf32 = False
    cfg, w, m = synth_model("arctic")
    ids, cu = synth.make_inputs("c3")
    got = m.encode_packed(ids, cu)
    ref = TorchRef(cfg, w, device="cuda")
    want = ref.encode_packed(ids, cu)
    del ref
    torch.cuda.empty_cache()
    assert_parity(got, want, "c3-full")


def test_c3_q8_full_vs_oracle(gpu):
    """c3 int8 path at full size (16 × 2048, the long-context + fused
    dequantise-GEMM stress case) against the oracle's Q8 forward on every
    host core: every vector bit-identical."""
    gemm = _q8_oracle_or_skip()
    cfg, w, m = synth_model("arctic", q8=True)
    ids, cu = synth.make_inputs("c3")
    got = m.encode_packed(ids, cu)
    want = OracleModel(cfg, w, q8=True, gemm=gemm).encode_batch(ids, cu)
    same = int(np.sum(np.all(got == want, axis=1)))
    print(f"[q8] c3-full: {same}/{len(got)} vectors bit-identical")
    assert_parity(got, want, "c3-full q8", Q8_COSINE_MIN)
    assert same == len(got)


# ---------------------------------------------------------------------------
# Invariants: batch ≡ single, determinism, device-resident entry point
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("arch,inputs,nseq,layers", [
    ("bge", "c0", 32, None),       # CLS pooling: the pruned last layer splits too
    ("minilm6", "c1", 16, None),   # mean pooling, 128-token sequences (two key tiles)
    ("nomic", "c2", 4, 3),         # head_dim 64, one head per step, up to 512 tokens
    ("bge", "c4", 64, 2),          # head_dim 32 with sequences past 128 tokens
])
def test_attention_split_bitwise_equals_unsplit(gpu, monkeypatch, arch, inputs, nseq, layers):
    """Small micro-batches spread each attention tile's head groups over
    several CTAs (the default); every head is computed by the same code in
    the same order, so the vectors equal the one-CTA-per-tile ones bit for
    bit (FUTON_CUDA_ATTN_SPLIT=0)."""
    cfg = synth.arch(arch)
    if layers:
        cfg.num_layers = layers
    w = synth.make_weights(cfg)
    ids, cu = synth.make_inputs(inputs, nseq=nseq, vocab=cfg.vocab_size)
    out = {}
    for v in ("1", "0"):
        monkeypatch.setenv("FUTON_CUDA_ATTN_SPLIT", v)
        m = Model(cfg, w, devices=[0])
        out[v] = m.encode_packed(ids, cu)
        m.close()
    assert np.array_equal(out["1"], out["0"])


@pytest.mark.parametrize("arch,inputs,nseq", [
    ("bge", "c4", 700),      # M-tail tiles, the fused LayerNorm clusters
    ("nomic", "c2", 24),     # SwiGLU fc1‖gate, RoPE qkv
])
def test_gemm_pair_tiles_match_single_cta(gpu, monkeypatch, arch, inputs, nseq):
    """CTA-pair GEMM tiles (FUTON_CUDA_GEMM_PAIR=1: M = 256 over two SMs with
    cta_group::2 MMAs, each CTA staging half of the weight tile) against the
    default one CTA per 128-row tile: the same products summed over the same
    k-blocks, so the vectors are bit-identical, and both meet the oracle gate."""
    cfg = synth.arch(arch)
    w = synth.make_weights(cfg)
    ids, cu = synth.make_inputs(inputs, nseq=nseq, vocab=cfg.vocab_size)
    out = {}
    for v in ("1", "0"):
        monkeypatch.setenv("FUTON_CUDA_GEMM_PAIR", v)
        m = Model(cfg, w, devices=[0])
        out[v] = m.encode_packed(ids, cu)
        m.close()
    assert np.array_equal(out["1"], out["0"])
    n = min(nseq, 64)
    want = OracleModel(cfg, w, gemm=oracle_mode()).encode_batch(ids[:cu[n]], cu[:n + 1])
    assert_parity(out["1"][:n], want, f"pair tiles {arch}")


def test_batch_matches_single_bitwise(gpu):
    """Packing never perturbs a sequence (no padding, no cross-sequence
    reduction): each vector of a packed call equals its single-sequence call."""
    cfg, w, m = synth_model("bge")
    ids, cu = synth.make_inputs("c4", nseq=40, seed=3)
    batch = m.encode_packed(ids, cu)
    for i in range(len(cu) - 1):
        single = m.encode_tokens(ids[cu[i]:cu[i + 1]])
        assert np.array_equal(single, batch[i]), f"sequence {i} differs"


def test_deterministic_runs(gpu):
    cfg, w, m = synth_model("nomic")
    ids, cu = synth.make_inputs("c2", nseq=8, seed=4)
    a = m.encode_packed(ids, cu, out_dim=256)
    b = m.encode_packed(ids, cu, out_dim=256)
    assert np.array_equal(a, b)


def test_concurrent_callers(gpu):
    """Model is safe for concurrent use (native/model.go:14-15): host threads
    calling into one model at once get exactly their serial results (calls on
    a device are serialised inside the library)."""
    import threading
    cfg, w, m = synth_model("bge")
    batches = [synth.make_inputs("c4", nseq=64 + 16 * i, seed=20 + i) for i in range(4)]
    want = [m.encode_packed(ids, cu) for ids, cu in batches]
    got = [None] * len(batches)
    errors = []

    def run(i):
        try:
            for _ in range(3):
                got[i] = m.encode_packed(*batches[i])
        except Exception as e:  # surfaced below
            errors.append(e)

    threads = [threading.Thread(target=run, args=(i,)) for i in range(len(batches))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    for g, w_ in zip(got, want):
        assert np.array_equal(g, w_)


def test_encode_device_matches_host(gpu):
    import torch
    cfg, w, m = synth_model("bge")
    ids, cu = synth.make_inputs("c4", nseq=300, seed=7)
    host = m.encode_packed(ids, cu)
    d_ids = torch.from_numpy(ids).cuda()
    d_out = torch.empty((len(cu) - 1, cfg.hidden_size), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    m.encode_device(d_ids.data_ptr(), cu, 0, d_out.data_ptr(), stream=s.cuda_stream)
    m.sync(stream=s.cuda_stream)
    assert np.array_equal(d_out.cpu().numpy(), host)
    assert m.launch_count() > 0


def test_graph_replay_takes_each_calls_batch(gpu):
    """Small host-buffer calls run from a CUDA graph captured by the first call
    with the same launches and replayed after this call's ids and tile lists
    are uploaded: a repeated batch, the same sequences in another order (same
    shape: same token count, sequence count and tiles) and other token ids
    with the same lengths each give their own vectors, bit for bit the ones
    of the device-resident entry point (which launches directly)."""
    import torch
    from futon_b200 import pack_ids
    cfg, w, m = synth_model("bge")
    ids, cu = synth.make_inputs("c0", nseq=32, seed=21)
    a = m.encode_packed(ids, cu)
    assert np.array_equal(m.encode_packed(ids, cu), a)
    perm = np.arange(len(cu) - 1)[::-1]
    ids_b, cu_b = pack_ids([ids[cu[i]:cu[i + 1]] for i in perm])
    assert np.array_equal(m.encode_packed(ids_b, cu_b), a[perm])
    ids_c = np.random.default_rng(3).integers(1000, cfg.vocab_size, ids.size).astype(np.int32)
    c = m.encode_packed(ids_c, cu)
    d_ids = torch.from_numpy(ids_c).cuda()
    d_out = torch.empty((len(cu) - 1, cfg.hidden_size), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    m.encode_device(d_ids.data_ptr(), cu, 0, d_out.data_ptr(), stream=s.cuda_stream)
    m.sync(stream=s.cuda_stream)
    assert np.array_equal(d_out.cpu().numpy(), c)
    assert not np.array_equal(c, a)


def test_io_bytes_counts_the_copies(gpu):
    """futon_cuda_io_bytes: a host-buffer call copies at least the ids in and
    exactly the vectors plus the 4-byte device error word out."""
    cfg, w, m = synth_model("bge")
    ids, cu = synth.make_inputs("c0", seed=13)
    h0, d0 = m.io_bytes()
    m.encode_packed(ids, cu)
    h1, d1 = m.io_bytes()
    assert h1 - h0 >= ids.nbytes + cu.nbytes
    assert d1 - d0 == (len(cu) - 1) * cfg.hidden_size * 4 + 4


def test_encode_device_two_streams(gpu):
    """Back-to-back device-resident calls on two different caller streams,
    queued without waiting, share the device's workspace: the library orders
    the second after the first, so both match the host-buffer path."""
    import torch
    cfg, w, m = synth_model("bge")
    batches = [synth.make_inputs("c4", nseq=400, seed=11), synth.make_inputs("c0", seed=12)]
    want = [m.encode_packed(ids, cu) for ids, cu in batches]
    d_ids = [torch.from_numpy(ids).cuda() for ids, _ in batches]
    d_out = [torch.empty((len(cu) - 1, cfg.hidden_size), dtype=torch.float32, device="cuda")
             for _, cu in batches]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for (ids, cu), di, do, s in zip(batches, d_ids, d_out, streams):
        m.encode_device(di.data_ptr(), cu, 0, do.data_ptr(), stream=s.cuda_stream)
    for s in streams:
        m.sync(stream=s.cuda_stream)
    for do, wv in zip(d_out, want):
        assert np.array_equal(do.cpu().numpy(), wv)


def test_micro_batching_large_call(gpu):
    """A call larger than one micro-batch (524,288 tokens) splits without
    changing any vector."""
    cfg, w, m = synth_model("bge")
    ids, cu = synth.make_inputs("c4", nseq=7000, seed=9)
    assert cu[-1] > 524288
    big = np.concatenate([ids] * 1)
    full = m.encode_packed(big, cu)
    # re-encode a slice that crosses no boundary and compare
    sub = m.encode_packed(ids[cu[100]:cu[140]], cu[100:141] - cu[100])
    assert np.array_equal(full[100:140], sub)
    n = np.linalg.norm(full, axis=1)
    assert np.abs(n - 1).max() <= NORM_TOL


# ---------------------------------------------------------------------------
# Rejects and cancellation (model_test.go:416-471, 203-244)
# ---------------------------------------------------------------------------
def test_rejects(gpu):
    p = load_pack(GOLDEN / "toy-absolute-gelu")
    m = Model(p.cfg, p.tensors, devices=[0])
    with pytest.raises(FutonError, match="empty"):
        m.encode_tokens([])
    with pytest.raises(FutonError, match="outside vocab"):
        m.encode_tokens([2, 999, 3])
    with pytest.raises(FutonError, match="exceeds effective max_seq_len"):
        m.encode_tokens([5] * (p.cfg.max_seq_len + 1))
    with pytest.raises(FutonError, match="matryoshka"):
        m.encode_tokens([2, 3], 16)
    with pytest.raises(FutonError, match="outside"):
        m.encode_tokens([2, 3], p.cfg.hidden_size + 1)
    with pytest.raises(FutonError, match="empty"):
        m.encode_packed(np.array([2, 3], np.int32), np.array([0, 2, 2], np.int32))
    with pytest.raises(FutonError, match="null buffer"):  # caught on the host, nothing launched
        m.encode_device(0, np.array([0, 2], np.int32), 0, 0)
    m.close()


def test_cancellation(gpu):
    cfg, w, m = synth_model("bge")
    ids, cu = synth.make_inputs("c0")
    flag = CancelFlag()
    flag.cancel()
    with pytest.raises(CanceledError):
        m.encode_packed(ids, cu, cancel=flag)
    # The model stays usable after a canceled call.
    out = m.encode_packed(ids, cu)
    assert np.abs(np.linalg.norm(out, axis=1) - 1).max() <= NORM_TOL


def test_cancellation_at_every_checkpoint(gpu):
    """Cancellation at each checkpoint of a two-micro-batch call, like the
    reference's cancelAfterN context (model_test.go:203-244): the call
    returns the cancel error, writes no vector, and the next call is
    bit-identical to a clean run."""
    from futon_b200 import _lib, pack_ids
    cfg = synth.arch("bge")
    cfg.num_layers = 2
    w = synth.make_weights(cfg)
    m = Model(cfg, w, devices=[0])
    seqs = [np.full(128, 1000 + i % 7, np.int32) for i in range(4200)]  # 537,600 tokens
    ids, cu = pack_ids(seqs)
    clean = m.encode_packed(ids, cu)
    # Checkpoints: the entry check, then per micro-batch (two of ≤ 524,288
    # tokens) one before it, and one before each layer and each layer's FFN.
    checkpoints = 1 + 2 * (1 + 2 * cfg.num_layers)
    lib = _lib.lib()
    try:
        for k in range(checkpoints):
            out = np.full((len(seqs), cfg.hidden_size), np.nan, np.float32)
            lib.futon_cuda_debug_cancel_after(k)
            with m._call() as h, pytest.raises(CanceledError):
                _lib.call("futon_cuda_encode", h, 0, ids.ctypes.data, cu.ctypes.data, len(seqs), 0,
                          out.ctypes.data, None)
            assert np.isnan(out).all(), f"checkpoint {k}: a partial vector was written"
            again = m.encode_packed(ids, cu)
            assert np.array_equal(again, clean), f"checkpoint {k}: the next call differs"
        # With as many passes as checkpoints the call completes.
        lib.futon_cuda_debug_cancel_after(checkpoints)
        assert np.array_equal(m.encode_packed(ids, cu), clean)
    finally:
        lib.futon_cuda_debug_cancel_after(-1)
        m.close()


def test_trained_context_clamp(gpu):
    """Sequences past max_trained_positions are refused (config.go:111-116)."""
    import copy
    p = load_pack(GOLDEN / "toy-rope-swiglu")
    cfg = copy.deepcopy(p.cfg)
    cfg.max_trained_positions = 16
    m = Model(cfg, p.tensors, devices=[0])
    m.encode_tokens([5] * 16)
    with pytest.raises(FutonError, match="exceeds effective max_seq_len 16"):
        m.encode_tokens([5] * 17)
    m.close()
