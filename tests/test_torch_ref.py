"""Pins the plain-PyTorch restatement (tests/torch_ref.py) to the CPU oracle
on the CPU, so the GPU tests may use it where the scalar oracle is too slow
(full-size c3 at L = 2048)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN, row_cosines
from futon_b200 import synth
from futon_b200.pack import load_pack
from oracle.oracle import GEMM_AVX2, GEMM_GO, OracleModel, has_avx2
from torch_ref import TorchRef


@pytest.mark.parametrize("pack", ["toy-absolute-gelu", "toy-rope-swiglu"])
def test_toy_matches_oracle(pack, toy_expected):
    pk = load_pack(GOLDEN / pack, keep_f16=False)
    ref = TorchRef(pk.cfg, pk.tensors, dtype=torch.float64)
    o = OracleModel(pk.cfg, pk.tensors)
    for c in toy_expected["packs"][pack]["forward_cases"]:
        a, b = ref.encode(c["ids"]), o.encode(c["ids"])
        assert np.abs(a - b).max() <= 1e-5
    for c in toy_expected["packs"][pack].get("matryoshka_cases", []):
        a, b = ref.encode(c["ids"], c["dim"]), o.encode(c["ids"], c["dim"])
        assert np.abs(a - b).max() <= 1e-5


@pytest.mark.parametrize("arch", ["bge", "arctic"])
def test_small_arch_matches_oracle(arch):
    """2-layer versions of the benchmark architectures at L up to 96."""
    cfg = synth.arch(arch)
    cfg.num_layers = 2
    w = synth.make_weights(cfg)
    rng = np.random.default_rng(2)
    seqs = [np.concatenate([[101], rng.integers(1000, cfg.vocab_size, L - 2), [102]])
            for L in (9, 40, 96)]
    cu = np.concatenate([[0], np.cumsum([len(s) for s in seqs])]).astype(np.int32)
    ids = np.concatenate(seqs).astype(np.int32)
    want = OracleModel(cfg, w, gemm=GEMM_AVX2 if has_avx2() else GEMM_GO).encode_batch(ids, cu)
    got = TorchRef(cfg, w, dtype=torch.float32).encode_packed(ids, cu)
    assert row_cosines(got, want).min() >= 0.999999


def test_q8_emulation_matches_oracle():
    """The float64 Q8 emulation agrees with the oracle's Q8 forward on a
    1-layer arctic shape (bit-level agreement is not expected; see
    tests/study_q8_sensitivity.py)."""
    cfg = synth.arch("arctic")
    cfg.num_layers = 1
    w = synth.make_weights(cfg)
    rng = np.random.default_rng(4)
    seqs = [np.concatenate([[101], rng.integers(1000, cfg.vocab_size, L - 2), [102]]) for L in (17, 64)]
    cu = np.concatenate([[0], np.cumsum([len(s) for s in seqs])]).astype(np.int32)
    ids = np.concatenate(seqs).astype(np.int32)
    want = OracleModel(cfg, w, q8=True).encode_batch(ids, cu)
    got = TorchRef(cfg, w, dtype=torch.float64, q8=True).encode_packed(ids, cu)
    assert row_cosines(got, want).min() >= 0.9999
