"""GPU checks of the opt-in attention variants, selected when a model is
created by FUTON_CUDA_ATTN / FUTON_CUDA_ATTN_SPLIT.

These run only on request (`FUTON_TEST_ATTN_VARIANTS=1 pytest -m
gpu_variant`): the default configuration never reaches the variants, so the
default `-m gpu` suite does not select them.

- split: attn_heads_kernel with the head groups shared among grid.y CTAs.
  Every head is computed by the same code in the same order as without the
  split, so the vectors must be bitwise equal to the default kernel's.
- tc, tc2: the tcgen05 attention kernels (tc2: separate q·k and v rings
  and two softmax warpgroups; head_dim 32 or 64 with an even head count);
  parity with the oracle (cosine gate) and batch invariance (a sequence's
  vector does not depend on what it is packed with).
- FUTON_CUDA_Q8_ATTN=exact: the int8 path's attention in the reference's
  exact float32 operation order (avx2Kernel MatMulT, softmaxScaled); its
  arithmetic is checked bit for bit on the CPU by test_exact_host.py.
  On the GPU the int8 forward must then sit within float32 noise of the
  oracle's int8 forward (avx2Kernel order), far inside the 0.9999 gate.
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


@pytest.mark.parametrize("arch,inputs,nseq,layers", CASES)
def test_split_bitwise_equals_default(gpu, monkeypatch, arch, inputs, nseq, layers):
    cfg, w = weights(arch, layers)
    ids, cu = synth.make_inputs(inputs, nseq=nseq, vocab=cfg.vocab_size)
    base = encode(monkeypatch, {}, cfg, w, ids, cu)
    split = encode(monkeypatch, {"FUTON_CUDA_ATTN_SPLIT": "1"}, cfg, w, ids, cu)
    assert np.array_equal(base, split), f"{arch}: split attention differs from the default"


@pytest.mark.parametrize("kernel", ["tc", "tc2"])
@pytest.mark.parametrize("arch,inputs,nseq,layers", CASES)
def test_tc_vs_oracle(gpu, monkeypatch, kernel, arch, inputs, nseq, layers):
    cfg, w = weights(arch, layers)
    ids, cu = synth.make_inputs(inputs, nseq=nseq, vocab=cfg.vocab_size)
    got = encode(monkeypatch, {"FUTON_CUDA_ATTN": kernel}, cfg, w, ids, cu)
    gemm = GEMM_AVX2 if has_avx2() else GEMM_GO
    want = OracleModel(cfg, w, gemm=gemm).encode_batch(ids, cu)
    cs = row_cosines(got, want)
    assert cs.min() >= GPU_COSINE_MIN, f"{arch}: {kernel} attention min cosine {cs.min():.7f}"


@pytest.mark.parametrize("kernel", ["tc", "tc2"])
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
    ("nomic", "c2", 4, 2),    # mean pooling: every layer attends over all rows
])
def test_q8_exact_attention_vs_oracle(gpu, monkeypatch, arch, inputs, nseq, layers):
    if not has_avx2():
        pytest.skip("the oracle's avx2Kernel order needs an AVX2 host")
    cfg, w = weights(arch, layers)
    ids, cu = synth.make_inputs(inputs, nseq=nseq, vocab=cfg.vocab_size)
    got = encode(monkeypatch, {"FUTON_CUDA_Q8_ATTN": "exact"}, cfg, w, ids, cu, q8=True)
    want = OracleModel(cfg, w, q8=True, gemm=GEMM_AVX2).encode_batch(ids, cu)
    cs = row_cosines(got, want)
    same = int(np.sum(np.all(got == want, axis=1)))
    print(f"[q8 exact] {arch}: min cos {cs.min():.9f}, {same}/{len(cs)} vectors bit-identical")
    assert cs.min() >= 0.99999, f"{arch}: exact int8 attention min cosine {cs.min():.9f}"
