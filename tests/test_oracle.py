"""CPU oracle pinned against the reference's own tests and golden vectors.

Mirrors native/model_test.go (toy forward goldens, determinism, batch ≡
single, rejects, trained-context clamp), native/kernel_test.go (GEMM vs a
float64 naive reference), native/quant_test.go (Q8 primitives, exact Q8
GEMM, toy Q8 forward) and native/mathf32_test.go (accuracy bounds).
"""
from __future__ import annotations

import copy
import hashlib
import json
import math

import numpy as np
import pytest

from conftest import GOLDEN, TOY_ABS_TOL, TOY_COSINE_MIN, cosine
from futon_b200 import pack_ids, synth
from futon_b200.pack import load_pack
from oracle import oracle as O

PACKS = ("toy-absolute-gelu", "toy-rope-swiglu")


@pytest.fixture(scope="module")
def toy_models():
    out = {}
    for p in PACKS:
        pk = load_pack(GOLDEN / p, keep_f16=False)
        out[p] = (pk, O.OracleModel(pk.cfg, pk.tensors))
    return out


def assert_close(got, want, label):
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, label
    assert cosine(got, want) >= TOY_COSINE_MIN, f"{label}: cosine {cosine(got, want)}"
    assert np.abs(got - want).max() <= TOY_ABS_TOL, f"{label}: max |d| {np.abs(got - want).max()}"


def test_golden_fixture_checksums():
    sums = json.loads((GOLDEN / "SHA256SUMS.json").read_text())
    for rel, digest in sums.items():
        assert hashlib.sha256((GOLDEN / rel).read_bytes()).hexdigest() == digest, rel


def test_toy_forward_goldens(toy_models, toy_expected):
    """TestToyForward (model_test.go:72-99): both option sets vs upstream."""
    for pack, pexp in toy_expected["packs"].items():
        _, m = toy_models[pack]
        for i, c in enumerate(pexp["forward_cases"]):
            assert_close(m.encode(c["ids"]), c["vector"], f"{pack} case {i}")
        for c in pexp.get("matryoshka_cases", []):
            got = m.encode(c["ids"], c["dim"])
            assert got.shape == (c["dim"],)
            assert_close(got, c["vector"], f"{pack} matryoshka")
        for c in pexp.get("text_cases", []):
            assert_close(m.encode(c["ids"]), c["vector"], f"{pack} text {c['text']!r}")


def test_oracle_regression_vectors(toy_models):
    """Bit-exact against the oracle's own recorded outputs (a regression pin)."""
    rec = json.loads((GOLDEN / "oracle_vectors.json").read_text())
    for pack, r in rec.items():
        _, m = toy_models[pack]
        for c in r["forward_cases"]:
            assert np.array_equal(m.encode(c["ids"]), np.asarray(c["vector"], np.float32))
        for c in r["matryoshka_cases"]:
            assert np.array_equal(m.encode(c["ids"], c["dim"]), np.asarray(c["vector"], np.float32))


def test_determinism_and_batch_equals_single(toy_models):
    """TestDeterminism / TestBatchMatchesSingle (model_test.go:127-197)."""
    _, m = toy_models["toy-rope-swiglu"]
    seqs = [[2, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 17, 3], [2, 3], [2] + [5] * 40 + [3]]
    ids, cu = pack_ids(seqs)
    singles = [m.encode(s) for s in seqs]
    for threads in (1, 2, 4):
        batch = m.encode_batch(ids, cu, threads=threads)
        for i, s in enumerate(singles):
            assert np.array_equal(batch[i], s)


def test_rejects(toy_models):
    """TestModelRejects (model_test.go:416-439)."""
    pk, m = toy_models["toy-absolute-gelu"]
    with pytest.raises(O.OracleError, match="empty"):
        m.encode([])
    with pytest.raises(O.OracleError, match="outside vocab"):
        m.encode([2, 999, 3])
    with pytest.raises(O.OracleError, match="exceeds"):
        m.encode([0] * (pk.cfg.max_seq_len + 1))
    with pytest.raises(O.OracleError, match="matryoshka"):
        m.encode([2, 3], 16)
    with pytest.raises(O.OracleError, match="outside"):
        m.encode([2, 3], pk.cfg.hidden_size + 1)


def test_trained_context_clamp():
    """TestTrainedContextClamp (model_test.go:252-300): past the trained
    context the model refuses; at it, it runs."""
    pk = load_pack(GOLDEN / "toy-rope-swiglu", keep_f16=False)
    cfg = copy.deepcopy(pk.cfg)
    cfg.max_trained_positions = 16
    assert cfg.effective_max_seq_len() == 16
    m = O.OracleModel(cfg, pk.tensors)
    m.encode([5] * 16)
    with pytest.raises(O.OracleError, match="exceeds effective max_seq_len 16"):
        m.encode([5] * 17)


# ---- kernel_test.go -----------------------------------------------------------
SHAPES = [(1, 1, 1), (1, 7, 5), (3, 4, 9), (4, 4, 4), (5, 3, 8), (7, 16, 33), (8, 8, 64),
          (13, 29, 17), (32, 6, 100)]


@pytest.mark.parametrize("avx2", [False, True])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_vs_naive(m, n, k, avx2):
    rng = np.random.default_rng(42 + m * 100 + n * 10 + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    want = a.astype(np.float64) @ b.astype(np.float64).T + bias
    got = O.matmul_t(a, b, bias, avx2=avx2)
    assert np.abs(got - want).max() <= 1e-4


def test_gemm_summation_order_is_gokernel():
    """The scalar oracle sums each 4-chunk as ((a0b0 + a1b1) + a2b2) + a3b3,
    then the tail, then the bias (kernel.go:239-259)."""
    rng = np.random.default_rng(7)
    a = rng.standard_normal((3, 11)).astype(np.float32)
    b = rng.standard_normal((2, 11)).astype(np.float32)
    bias = rng.standard_normal(2).astype(np.float32)
    got = O.matmul_t(a, b, bias)
    for i in range(3):
        for j in range(2):
            s = np.float32(0)
            p = 0
            while p + 4 <= 11:
                t = np.float32(a[i, p] * b[j, p]) + np.float32(a[i, p + 1] * b[j, p + 1])
                t = np.float32(t + np.float32(a[i, p + 2] * b[j, p + 2]))
                t = np.float32(t + np.float32(a[i, p + 3] * b[j, p + 3]))
                s = np.float32(s + t)
                p += 4
            for q in range(p, 11):
                s = np.float32(s + np.float32(a[i, q] * b[j, q]))
            s = np.float32(s + bias[j])
            assert got[i, j] == s


# ---- quant_test.go -----------------------------------------------------------
def test_q8_quantize_row():
    rng = np.random.default_rng(3)
    src = rng.standard_normal((1, 257)).astype(np.float32)
    q, s = O.quantize_rows_q8(src)
    amax = np.abs(src).max()
    assert s[0] > 0 and abs(float(s[0]) - amax / 127) <= 1e-6 * amax
    assert (q != -128).all()
    err = np.abs(src[0].astype(np.float64) - q[0].astype(np.float64) * float(s[0]))
    assert (err <= float(s[0]) / 2 + 1e-7).all()
    qz, sz = O.quantize_rows_q8(np.zeros((1, 8), np.float32))
    assert sz[0] == 0 and (qz == 0).all()


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (2, 3, 7), (4, 4, 8), (5, 9, 16), (7, 16, 33),
                                   (13, 29, 65)])
def test_q8_matmul_exact(m, n, k):
    rng = np.random.default_rng(17 + m + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    qb, sb = O.quantize_rows_q8(w)
    qa, sa = O.quantize_rows_q8(a)
    acc = qa.astype(np.int64) @ qb.astype(np.int64).T
    want = (acc.astype(np.float32) * (sa[:, None] * sb[None, :])).astype(np.float32) + bias
    got = O.matmul_t_q8(a, qb, sb, bias)
    assert np.array_equal(got, want.astype(np.float32))


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (3, 5, 15), (4, 7, 16), (9, 33, 100), (64, 96, 768),
                                   (17, 40, 3072)])
def test_q8_prequant_avx2_equals_scalar(m, n, k):
    """The oracle's AVX2 int8 dot gives the reference loop's exact sums: the
    two prequantised GEMMs agree bit for bit, extremes (±127 everywhere,
    the largest possible sums) included."""
    rng = np.random.default_rng(m * 1000 + n + k)
    qa = rng.integers(-127, 128, size=(m, k), dtype=np.int64).astype(np.int8)
    qb = rng.integers(-127, 128, size=(n, k), dtype=np.int64).astype(np.int8)
    qa[0, :] = -127
    qb[0, :] = -127
    sa = rng.random(m).astype(np.float32)
    sb = rng.random(n).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    out = {}
    for name in ("fo_matmul_t_q8_prequant", "fo_matmul_t_q8_prequant_scalar"):
        o = np.zeros((m, n), np.float32)
        getattr(O.lib(), name)(o.ctypes.data, qa.ctypes.data, sa.ctypes.data, qb.ctypes.data,
                               sb.ctypes.data, m, n, k, bias.ctypes.data)
        out[name] = o
    a, b = out.values()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_q8_toy_forward(toy_expected):
    """TestQ8ToyForward (quant_test.go:152-183): Q8 tracks the goldens ≥ 0.98."""
    for pack, pexp in toy_expected["packs"].items():
        pk = load_pack(GOLDEN / pack, keep_f16=False)
        m = O.OracleModel(pk.cfg, pk.tensors, q8=True)
        assert m.q8_weight(0, 0) is not None
        for c in pexp["forward_cases"]:
            assert cosine(m.encode(c["ids"]), c["vector"]) >= 0.98


# ---- mathf32_test.go ---------------------------------------------------------
def test_math_accuracy():
    xs = np.arange(-87.33654 + 0.01, 88.72283 - 0.01, 0.0731, dtype=np.float64).astype(np.float32)
    rel = max(abs(O.exp_f32(float(x)) - math.exp(float(x))) / math.exp(float(x)) for x in xs)
    assert rel <= 2 ** -23
    assert O.exp_f32(0.0) == 1.0 and O.exp_f32(-104.0) == 0.0
    gx = np.arange(-12, 12, 0.0117, dtype=np.float32)
    gerr = max(abs(O.gelu_f32(float(x)) - 0.5 * float(x) * (1 + math.erf(float(x) / math.sqrt(2))))
               for x in gx)
    assert gerr <= 1e-6
    sx = np.arange(-120, 120, 0.0913, dtype=np.float32)
    serr = max(abs(O.sigmoid_f32(float(x)) - 1 / (1 + math.exp(-float(x)))) for x in sx)
    assert serr <= 2e-7


def test_synthetic_config_flops():
    """The benchmark's FLOP accounting (c1 is exact: 256 × 128 tokens)."""
    cfg = synth.arch("minilm6")
    ids, cu = synth.make_inputs("c1")
    assert int(cu[-1]) == 32768
    assert abs(synth.total_flops(cfg, cu) / 1e12 - 0.7344) < 1e-3
