"""Synthetic packs and inputs for the benchmark configurations.

Architectures follow the reference's pack configs (scripts/build-weight-pack.py
NOMIC_CONFIG / ARCTIC_CONFIG / BGE_CONFIG) at random-init weights: every
matrix, embedding table and bias ~ N(0, 0.02) from numpy default_rng(seed),
LayerNorm γ = 1 and β = 0 (nomic-bert shapes carry no linear biases).
Inputs: each sequence is [CLS]=101, uniform ids in [1000, vocab-1], [SEP]=102,
so a sequence's length includes both special tokens.

  c0  bge-small shape, 32 sequences, L ~ U[8, 128], CLS pooling
  c1  MiniLM-L6 shape, 256 × 128, mean pooling
  c2  nomic-bert shape, 64 sequences, L ~ U[64, 512], mean pooling,
      matryoshka 768/256/64
  c3  arctic-embed-m-long shape, 16 × 2048, CLS pooling, fp32 and Q8
  c4  bge-small shape, 65,536 sequences, L = clip(round(exp(ln 64 + 0.8 N)), 8, 512)

Text inputs (make_texts) stand in for a corpus where the tokenizer is part of
the path: each text is L-3 words drawn from the vocab's whole-word entries
plus a full stop, first word capitalised, so it tokenises to exactly L ids.
"""
from __future__ import annotations

import dataclasses
from typing import Dict, List, Optional, Tuple

import numpy as np

from .pack import Matryoshka, PackConfig, expected_tensor_shapes

CLS_ID, SEP_ID = 101, 102
TOKENIZER = {"cls_token": "[CLS]", "do_lower_case": True, "pad_token": "[PAD]",
             "sep_token": "[SEP]", "tokenize_chinese_chars": True, "unk_token": "[UNK]"}


def arch(name: str) -> PackConfig:
    """Architecture of a synthetic pack."""
    if name in ("bge", "minilm6"):
        return PackConfig(model_id="synthetic-bge-small" if name == "bge" else "synthetic-minilm-l6",
                          hidden_size=384, num_layers=12 if name == "bge" else 6, num_heads=12,
                          intermediate_size=1536, vocab_size=30522, type_vocab_size=2,
                          max_seq_len=512, layer_norm_eps=1e-12, position_encoding="absolute",
                          activation="gelu", pooling="cls" if name == "bge" else "mean",
                          normalize=True, tokenizer=dict(TOKENIZER))
    if name in ("nomic", "arctic"):
        return PackConfig(model_id="synthetic-nomic-bert" if name == "nomic" else "synthetic-arctic-m-long",
                          hidden_size=768, num_layers=12, num_heads=12, intermediate_size=3072,
                          vocab_size=30528, type_vocab_size=2, max_seq_len=8192,
                          layer_norm_eps=1e-12, position_encoding="rope", rope_theta=1000.0,
                          max_trained_positions=2048, activation="swiglu",
                          pooling="mean" if name == "nomic" else "cls", normalize=True,
                          matryoshka=(Matryoshka(layernorm=True, dims=[768, 512, 256, 128, 64])
                                      if name == "nomic" else None),
                          tokenizer=dict(TOKENIZER))
    raise KeyError(name)


@dataclasses.dataclass(frozen=True)
class BenchConfig:
    key: str
    arch: str
    nseq: int
    lengths: Tuple  # ("uniform", lo, hi) | ("fixed", L) | ("lognormal", median, sigma, lo, hi)
    out_dims: Tuple[int, ...] = (0,)
    q8_modes: Tuple[bool, ...] = (False,)


CONFIGS: Dict[str, BenchConfig] = {
    "c0": BenchConfig("c0", "bge", 32, ("uniform", 8, 128)),
    "c1": BenchConfig("c1", "minilm6", 256, ("fixed", 128)),
    "c2": BenchConfig("c2", "nomic", 64, ("uniform", 64, 512), out_dims=(768, 256, 64)),
    "c3": BenchConfig("c3", "arctic", 16, ("fixed", 2048), q8_modes=(False, True)),
    "c4": BenchConfig("c4", "bge", 65536, ("lognormal", 64, 0.8, 8, 512)),
    # The throughput target's shape: bge-small at sequence length 128.
    "bge-seq128": BenchConfig("bge-seq128", "bge", 8192, ("fixed", 128)),
}


def no_linear_biases(cfg: PackConfig) -> bool:
    # nomic-bert shapes (RoPE + SwiGLU) have no attention/FFN biases.
    return cfg.position_encoding == "rope" and cfg.activation == "swiglu"


def make_weights(cfg: PackConfig, seed: int = 0) -> Dict[str, np.ndarray]:
    """Random-init tensors in canonical names, generated in a fixed order."""
    rng = np.random.default_rng(seed)
    out: Dict[str, np.ndarray] = {}
    for name, shape in expected_tensor_shapes(cfg).items():
        is_bias = name.endswith(".bias") and ("norm" not in name)
        if is_bias and no_linear_biases(cfg):
            continue
        if "norm" in name:
            out[name] = (np.ones(shape, np.float32) if name.endswith("weight")
                         else np.zeros(shape, np.float32))
        else:
            out[name] = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
    return out


def sample_lengths(spec: Tuple, n: int, rng: np.random.Generator) -> np.ndarray:
    kind = spec[0]
    if kind == "uniform":
        return rng.integers(spec[1], spec[2] + 1, size=n)
    if kind == "fixed":
        return np.full(n, spec[1], dtype=np.int64)
    if kind == "lognormal":
        med, sigma, lo, hi = spec[1:]
        L = np.round(np.exp(np.log(med) + sigma * rng.standard_normal(n)))
        return np.clip(L, lo, hi).astype(np.int64)
    raise KeyError(kind)


def make_inputs(key: str, seed: int = 1, nseq: Optional[int] = None,
                vocab: Optional[int] = None) -> Tuple[np.ndarray, np.ndarray]:
    """Packed (ids int32, cu_seqlens int32) for a benchmark configuration."""
    bc = CONFIGS[key]
    cfg = arch(bc.arch)
    V = vocab or cfg.vocab_size
    n = bc.nseq if nseq is None else nseq
    rng = np.random.default_rng(seed)
    lens = sample_lengths(bc.lengths, n, rng)
    cu = np.zeros(n + 1, dtype=np.int32)
    np.cumsum(lens, out=cu[1:])
    ids = rng.integers(1000, V, size=int(cu[-1]), dtype=np.int64).astype(np.int32)
    ids[cu[:-1]] = CLS_ID
    ids[cu[1:] - 1] = SEP_ID
    return ids, cu


def make_texts(key: str, vocab_lines: List[str], seed: int = 1,
               nseq: Optional[int] = None) -> Tuple[List[str], np.ndarray]:
    """Synthetic texts with a configuration's lengths (in tokens, [CLS] and
    [SEP] included) over a WordPiece vocab; returns (texts, lengths)."""
    bc = CONFIGS[key]
    n = bc.nseq if nseq is None else nseq
    rng = np.random.default_rng(seed)
    lens = np.maximum(sample_lengths(bc.lengths, n, rng), 3)
    words = [w for w in vocab_lines if w.isascii() and w.isalpha() and w.islower()]
    if not words:
        raise ValueError("vocab has no whole-word entries")
    picks = rng.integers(0, len(words), size=int((lens - 3).sum()))
    texts, k = [], 0
    for L in lens:
        m = int(L) - 3
        body = " ".join(words[i] for i in picks[k:k + m])
        k += m
        texts.append(body[:1].upper() + body[1:] + ".")
    return texts, lens


def synthetic_vocab(cfg: PackConfig) -> List[str]:
    """vocab.txt with the BERT special tokens at their usual ids."""
    v = [f"[unused{i}]" for i in range(cfg.vocab_size)]
    v[0], v[100], v[101], v[102], v[103] = "[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"
    return v


def flops_per_sequence(cfg: PackConfig, L: int) -> float:
    """Algorithmic FLOPs of one forward (the work the reference performs):
    non-final layer 2L(4h² + (a+1)·inter·h) + 4L²h; with CLS pooling the
    final layer computes K/V for all rows but everything else for row 0."""
    h, I = cfg.hidden_size, cfg.intermediate_size
    a = 2 if cfg.activation == "swiglu" else 1
    full = 2.0 * L * (4 * h * h + (a + 1) * I * h) + 4.0 * L * L * h
    if cfg.pooling == "cls":
        last = 2.0 * L * 2 * h * h + 2 * h * h + 4.0 * L * h + 2.0 * (h * h + (a + 1) * I * h)
    else:
        last = full
    return (cfg.num_layers - 1) * full + last


def total_flops(cfg: PackConfig, cu: np.ndarray) -> float:
    lens = np.diff(cu).astype(np.float64)
    return float(sum(flops_per_sequence(cfg, int(L)) for L in lens))
