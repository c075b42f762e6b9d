"""CPU check of the int8 path's exact-order arithmetic against the oracle,
bit for bit: the attention (futon_b200/csrc/attn_exact.cuh) against the
oracle's attendHead (native/model.go:646-739) in the avx2Kernel summation
order, and the activations (futon_b200/csrc/mathf32.cuh: expF32, geluF32,
sigmoidF32, native/mathf32.go:40-120). Also the accuracy of the float
path's fast GELU formula against the exact-erf GELU.

tests/host/exact_host.cu runs the routines the device kernels call,
over the same 64-key tiles in the same order, as host code built with nvcc
(-ffp-contract=off). The device kernels add only the staging of those tiles.
"""
from __future__ import annotations

import ctypes as C
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def fx(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc not available to build the host harness")
    out = tmp_path_factory.mktemp("fx") / "libfx.so"
    cmd = [nvcc, "-O2", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
           "-Xcompiler", "-fPIC,-ffp-contract=off", "-I", str(ROOT / "futon_b200" / "csrc"),
           "-I", str(ROOT / "include"), "-o", str(out), str(ROOT / "tests" / "host" / "exact_host.cu")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    lib = C.CDLL(str(out))
    lib.fx_attend_head.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                   C.c_void_p]
    lib.fx_attend_head.restype = C.c_int
    for name in ("fx_exp_f32", "fx_gelu_f32", "fx_sigmoid_f32", "fx_gelu_fast_ref"):
        getattr(lib, name).argtypes = [C.c_float]
        getattr(lib, name).restype = C.c_float
    return lib


def needs_avx2():
    if not O.has_avx2():
        pytest.skip("the oracle's avx2Kernel order needs an AVX2 host")


@pytest.mark.parametrize("hd,h", [(32, 384), (64, 768)])
@pytest.mark.parametrize("seq", [1, 2, 7, 8, 9, 63, 64, 65, 128, 129, 257])
def test_exact_attention_bitwise(fx, hd, h, seq):
    needs_avx2()
    rng = np.random.default_rng(seq * 131 + hd)
    for rows in sorted({seq, 1}):
        qkv = (rng.standard_normal((seq, 3 * h)) * rng.uniform(0.1, 3.0)).astype(np.float32)
        head = int(rng.integers(0, h // hd))
        want = O.attend_head(qkv, hd, head, rows=rows, gemm=O.GEMM_AVX2)
        got = np.zeros((rows, hd), np.float32)
        assert fx.fx_attend_head(qkv.ctypes.data, seq, rows, h, hd, head, got.ctypes.data) == 0
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
            f"hd={hd} seq={seq} rows={rows}: max |diff| {np.abs(got - want).max():.3e}"


def test_exact_attention_large_scores(fx):
    """Scores far apart (the −104 clamp and underflowing exponents)."""
    needs_avx2()
    rng = np.random.default_rng(3)
    seq, h, hd = 80, 384, 32
    qkv = (rng.standard_normal((seq, 3 * h)) * 12.0).astype(np.float32)
    want = O.attend_head(qkv, hd, 5, gemm=O.GEMM_AVX2)
    got = np.zeros((seq, hd), np.float32)
    assert fx.fx_attend_head(qkv.ctypes.data, seq, seq, h, hd, 5, got.ctypes.data) == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_exp_f32_host_matches_oracle(fx):
    xs = np.concatenate([np.linspace(-104, 88.7, 20001, dtype=np.float32),
                         np.random.default_rng(0).uniform(-90, 88, 20000).astype(np.float32)])
    got = np.array([fx.fx_exp_f32(float(x)) for x in xs], np.float32)
    want = np.array([O.exp_f32(float(x)) for x in xs], np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _sweep():
    rng = np.random.default_rng(7)
    return np.concatenate([np.linspace(-12, 12, 60001, dtype=np.float32),
                           rng.standard_normal(60000).astype(np.float32) * 3,
                           np.float32([0.0, -0.0, 1e-30, -1e-30, 87.0, -87.0, 110.0, -110.0])])


@pytest.mark.parametrize("name,ref", [("fx_gelu_f32", "gelu_f32"), ("fx_sigmoid_f32", "sigmoid_f32")])
def test_activation_host_matches_oracle(fx, name, ref):
    xs = _sweep()
    f, r = getattr(fx, name), getattr(O, ref)
    got = np.array([f(float(x)) for x in xs], np.float32)
    want = np.array([r(float(x)) for x in xs], np.float32)
    bad = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
    assert bad.size == 0, f"{name}: {bad.size} mismatches, first at x={xs[bad[0]]!r}"


def test_fast_gelu_formula_error_bound(fx):
    """The float path's GELU (Abramowitz & Stegun 7.1.28 in gelu_fast2) stays
    within 7.1e-7 of the exact-erf GELU over [−12, 12] (float64 reference).
    The device evaluates the same formula with rcp.approx (within 1 ulp of
    the exact reciprocal used here), far below that bound."""
    import math
    xs = np.concatenate([np.linspace(-12, 12, 96001, dtype=np.float32),
                         np.linspace(3.9, 4.1, 20001, dtype=np.float32)])
    worst = 0.0
    for x in xs:
        x = float(x)
        exact = 0.5 * x * math.erfc(-x / math.sqrt(2.0))
        worst = max(worst, abs(fx.fx_gelu_fast_ref(x) - exact))
    assert worst <= 7.1e-7, worst
