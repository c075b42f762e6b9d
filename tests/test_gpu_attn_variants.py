"""GPU checks of the opt-in attention variants, selected when a model is
created by FUTON_CUDA_ATTN / FUTON_CUDA_Q8_ATTN.

These run only on request (`FUTON_TEST_ATTN_VARIANTS=1 pytest -m
gpu_variant`): the default configuration never reaches the variants, so the
default `-m gpu` suite does not select them.

- tc2: the tcgen05 attention kernel (separate q·k and v rings and two
  softmax warpgroups; head_dim 32 or 64 with an even head count);
  parity with the oracle (cosine gate) and batch invariance (a sequence's
  vector does not depend on what it is packed with).
- FUTON_CUDA_Q8_ATTN=split: the int8 path's split-precision tensor-core
  attention (bf16 hi + lo parts) instead of the default exact-order one.
  Not bit-identical to the reference's float32 order, so the per-row
  quantisations that follow amplify its float32-level differences: it is
  held to the reference's own Q8 acceptance rule against the float path
  (cos ≥ 0.999, native/quant.go:27-29) and to cos ≥ 0.9998 against the
  oracle's Q8 forward.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import GPU_COSINE_MIN, row_cosines
from futon_b200 import Model, pack_ids, synth
from oracle.oracle import GEMM_AVX2, GEMM_GO, OracleModel, has_avx2

pytestmark = [
    pytest.mark.gpu_variant,
    pytest.mark.skipif(os.environ.get("FUTON_TEST_ATTN_VARIANTS") != "1",
                       reason="opt-in: FUTON_TEST_ATTN_VARIANTS=1"),
]

_weights = {}


def weights(arch, layers=None):
    key = (arch, layers)
    if key not in _weights:
        cfg = synth.arch(arch)
        if layers:
            cfg.num_layers = layers
        _weights[key] = (cfg, synth.make_weights(cfg))
    return _weights[key]


def encode(monkeypatch, env, cfg, w, ids, cu, out_dim=0, q8=False):
    for k in ("FUTON_CUDA_ATTN", "FUTON_CUDA_ATTN_SPLIT", "FUTON_CUDA_Q8_ATTN"):
        monkeypatch.delenv(k, raising=False)
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    m = Model(cfg, w, devices=[0], q8=q8)
    try:
        return m.encode_packed(ids, cu, out_dim=out_dim)
    finally:
        m.close()


CASES = [
    ("bge", "c0", 32, None),       # CLS pooling: the pruned last layer splits too
    ("minilm6", "c1", 16, None),   # mean pooling, 128-token sequences (two key tiles)
    ("nomic", "c2", 4, 3),         # head_dim 64, one head per step, up to 512 tokens
    ("bge", "c4", 64, 2),          # head_dim 32 with sequences past 128 tokens (key blocks)
]


@pytest.mark.parametrize("kernel", ["tc2"])
@pytest.mark.parametrize("arch,inputs,nseq,layers", CASES)
def test_tc_vs_oracle(gpu, monkeypatch, kernel, arch, inputs, nseq, layers):
    cfg, w = weights(arch, layers)
    ids, cu = synth.make_inputs(inputs, nseq=nseq, vocab=cfg.vocab_size)
    got = encode(monkeypatch, {"FUTON_CUDA_ATTN": kernel}, cfg, w, ids, cu)
    gemm = GEMM_AVX2 if has_avx2() else GEMM_GO
    want = OracleModel(cfg, w, gemm=gemm).encode_batch(ids, cu)
    cs = row_cosines(got, want)
    assert cs.min() >= GPU_COSINE_MIN, f"{arch}: {kernel} attention min cosine {cs.min():.7f}"


@pytest.mark.parametrize("kernel", ["tc2"])
def test_tc_batch_invariance(gpu, monkeypatch, kernel):
    cfg, w = weights("bge", 2)
    ids, cu = synth.make_inputs("c4", nseq=24, vocab=cfg.vocab_size)
    seqs = [ids[cu[i]:cu[i + 1]] for i in range(len(cu) - 1)]
    env = {"FUTON_CUDA_ATTN": kernel}
    packed = encode(monkeypatch, env, cfg, w, ids, cu)
    rev_ids, rev_cu = pack_ids(seqs[::-1])
    rev = encode(monkeypatch, env, cfg, w, rev_ids, rev_cu)[::-1]
    assert np.array_equal(packed, rev), f"{kernel} attention: a vector depends on its batch neighbours"


@pytest.mark.parametrize("arch,inputs,nseq,layers", [
    ("arctic", "c3", 2, 3),   # RoPE, SwiGLU, CLS, head_dim 64, 2048 tokens
    ("bge", "c0", 16, None),  # absolute positions, GELU, CLS, head_dim 32
])
def test_q8_split_attention_vs_oracle(gpu, monkeypatch, arch, inputs, nseq, layers):
    if not has_avx2():
        pytest.skip("the oracle's avx2Kernel order needs an AVX2 host")
    cfg, w = weights(arch, layers)
    ids, cu = synth.make_inputs(inputs, nseq=nseq, vocab=cfg.vocab_size)
    got = encode(monkeypatch, {"FUTON_CUDA_Q8_ATTN": "split"}, cfg, w, ids, cu, q8=True)
    want = OracleModel(cfg, w, q8=True, gemm=GEMM_AVX2).encode_batch(ids, cu)
    flt = OracleModel(cfg, w, q8=False, gemm=GEMM_AVX2).encode_batch(ids, cu)
    cs, cf = row_cosines(got, want), row_cosines(got, flt)
    print(f"[q8 split] {arch}: min cos {cs.min():.9f} vs Q8 oracle, {cf.min():.9f} vs float")
    assert cs.min() >= 0.9998, f"{arch}: split int8 attention min cosine {cs.min():.9f}"
    assert cf.min() >= 0.999, f"{arch}: split int8 vs float min cosine {cf.min():.9f}"
