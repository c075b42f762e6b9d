"""Shared fixtures for the futon_b200 test suite.

Markers: `gpu` tests need a CUDA device and call libfuton_cuda through its
C ABI; `gpu_variant` tests check opt-in kernel variants on a GPU and run only
when FUTON_TEST_ATTN_VARIANTS=1; everything else runs on the CPU (oracle,
pack host logic, ABI loading, gloo multi-process planning).
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "toy"

# Reference gates (native/model_test.go:19-22) for the CPU oracle, and the
# north-star gate for the f16 tensor-core path.
TOY_COSINE_MIN = 0.99999
TOY_ABS_TOL = 2e-4
GPU_COSINE_MIN = 0.9999


def pytest_configure(config):
    # A checkout without the built library (it is not committed) builds it
    # once here; nvcc cross-compiles sm_100a without a GPU.
    from futon_b200 import build as fb_build
    if not fb_build.LIB.exists():
        fb_build.build()
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libfuton_cuda")
    config.addinivalue_line(
        "markers", "gpu_variant: GPU checks of opt-in kernel variants (FUTON_TEST_ATTN_VARIANTS=1)")


def cosine(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def row_cosines(a, b) -> np.ndarray:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


@pytest.fixture(scope="session")
def toy_expected():
    return json.loads((GOLDEN / "expected.json").read_text())


@pytest.fixture(scope="session")
def gpu():
    """Asserts a CUDA device and the built library are present (no skip: a
    GPU test that cannot reach the kernels must fail loudly)."""
    import futon_b200
    n = futon_b200.device_count()
    assert n > 0, "no CUDA device visible to libfuton_cuda"
    return n
