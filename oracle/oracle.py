"""ctypes bridge to the CPU oracle (liboracle.so, built from futon_oracle.c).

TEST INFRASTRUCTURE ONLY: the parity checker for libfuton_cuda. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference legs import
this module; the product path (futon_b200) never does.

The oracle restates the reference's forward (native/model.go:346-769), its
goKernel GEMM order (native/kernel.go:223-283), its float32 transcendentals
(native/mathf32.go) and its Q8 scheme (native/quant.go); see futon_oracle.h.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys
from pathlib import Path
from typing import Dict, Optional

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

G_WORD, G_POS, G_TYPE, G_EMB_NORM_W, G_EMB_NORM_B = range(5)
LAYER_SLOTS = ["attn.qkv.weight", "attn.qkv.bias", "attn.out.weight", "attn.out.bias",
               "norm1.weight", "norm1.bias", "mlp.fc1.weight", "mlp.fc1.bias",
               "mlp.gate.weight", "mlp.gate.bias", "mlp.fc2.weight", "mlp.fc2.bias",
               "norm2.weight", "norm2.bias"]
GLOBAL_SLOTS = ["embeddings.word", "embeddings.position", "embeddings.token_type",
                "embeddings.norm.weight", "embeddings.norm.bias"]
GEMM_GO, GEMM_AVX2 = 0, 1


class FoCfg(C.Structure):
    _fields_ = [("hidden", C.c_int), ("num_layers", C.c_int), ("num_heads", C.c_int),
                ("inter", C.c_int), ("vocab", C.c_int), ("type_vocab", C.c_int),
                ("max_seq_len", C.c_int), ("max_trained", C.c_int), ("eps", C.c_double),
                ("rope", C.c_int), ("rope_theta", C.c_double), ("swiglu", C.c_int),
                ("pool_mean", C.c_int), ("normalize", C.c_int), ("matryoshka", C.c_int),
                ("matryoshka_ln", C.c_int)]


def build() -> Path:
    """Compiles liboracle.so and libtokport.so (the tokenizer port) with the
    committed Makefile when either is stale."""
    gen = HERE.parent / "futon_b200" / "csrc" / "gen_unicode_tables.py"
    deps = {LIB: [HERE / "futon_oracle.c", HERE / "futon_oracle.h", HERE / "Makefile"],
            HERE / "libtokport.so": [HERE / "tokenizer_port.cpp", HERE / "Makefile", gen]}
    if any(not out.exists() or any(s.stat().st_mtime > out.stat().st_mtime for s in srcs)
           for out, srcs in deps.items()):
        subprocess.run(["make", "-s", "-C", str(HERE), f"PYTHON={sys.executable}"], check=True)
    return LIB


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(str(LIB))
        vp, ip, fp = C.c_void_p, C.c_int, C.c_float
        L.fo_create.restype = vp
        L.fo_create.argtypes = [C.POINTER(FoCfg), C.POINTER(vp), ip, ip, C.c_char_p, C.c_size_t]
        L.fo_destroy.argtypes = [vp]
        L.fo_encode.restype = ip
        L.fo_encode.argtypes = [vp, vp, ip, ip, vp, C.c_char_p, C.c_size_t]
        L.fo_encode_batch.restype = ip
        L.fo_encode_batch.argtypes = [vp, vp, vp, ip, ip, vp, ip, C.c_char_p, C.c_size_t]
        L.fo_q8_data.restype = vp
        L.fo_q8_data.argtypes = [vp, ip, ip]
        L.fo_q8_scale.restype = vp
        L.fo_q8_scale.argtypes = [vp, ip, ip]
        L.fo_effective_max_seq_len.restype = ip
        L.fo_effective_max_seq_len.argtypes = [vp]
        for name in ("fo_matmul_t", "fo_matmul_t_avx2"):
            getattr(L, name).argtypes = [vp, vp, vp, ip, ip, ip, vp]
        L.fo_quantize_row_q8.restype = fp
        L.fo_quantize_row_q8.argtypes = [vp, vp, ip]
        L.fo_matmul_t_q8.argtypes = [vp, vp, vp, vp, ip, ip, ip, vp]
        L.fo_matmul_t_q8_prequant.argtypes = [vp, vp, vp, vp, vp, ip, ip, ip, vp]
        L.fo_matmul_t_q8_prequant_scalar.argtypes = [vp, vp, vp, vp, vp, ip, ip, ip, vp]
        L.fo_layernorm_rows.argtypes = [vp, ip, ip, vp, vp, fp]
        L.fo_softmax_scaled.argtypes = [vp, ip, fp]
        for name in ("fo_exp", "fo_gelu", "fo_sigmoid"):
            getattr(L, name).restype = fp
            getattr(L, name).argtypes = [fp]
        L.fo_rope_tables.argtypes = [ip, ip, C.c_double, vp, vp]
        L.fo_has_avx2.restype = ip
        L.fo_attend_head.restype = ip
        L.fo_attend_head.argtypes = [vp, ip, ip, ip, ip, ip, vp, vp, ip, vp]
        _lib = L
    return _lib


class OracleError(RuntimeError):
    pass


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


class OracleModel:
    """A pack on the CPU oracle (one independent forward per sequence)."""

    def __init__(self, cfg, tensors: Dict[str, np.ndarray], q8: bool = False,
                 gemm: int = GEMM_GO):
        self.cfg = cfg
        c = FoCfg()
        c.hidden, c.num_layers, c.num_heads = cfg.hidden_size, cfg.num_layers, cfg.num_heads
        c.inter, c.vocab, c.type_vocab = cfg.intermediate_size, cfg.vocab_size, cfg.type_vocab_size
        c.max_seq_len, c.max_trained = cfg.max_seq_len, cfg.max_trained_positions
        c.eps = cfg.layer_norm_eps
        c.rope = 1 if cfg.position_encoding == "rope" else 0
        c.rope_theta = cfg.rope_theta
        c.swiglu = 1 if cfg.activation == "swiglu" else 0
        c.pool_mean = 1 if cfg.pooling == "mean" else 0
        c.normalize = 1 if cfg.normalize else 0
        c.matryoshka = 1 if cfg.matryoshka is not None else 0
        c.matryoshka_ln = 1 if (cfg.matryoshka is not None and cfg.matryoshka.layernorm) else 0
        self._keep = []
        names = list(GLOBAL_SLOTS)
        for i in range(cfg.num_layers):
            names += [f"layers.{i}.{s}" for s in LAYER_SLOTS]
        ptrs = (C.c_void_p * len(names))()
        for k, n in enumerate(names):
            if n in tensors:
                a = _f32(tensors[n])
                self._keep.append(a)
                ptrs[k] = a.ctypes.data
        err = C.create_string_buffer(512)
        self._h = lib().fo_create(C.byref(c), ptrs, 1 if q8 else 0, gemm, err, 512)
        if not self._h:
            raise OracleError(err.value.decode())
        self.q8 = q8

    def close(self):
        if self._h:
            lib().fo_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def out_width(self, out_dim: int) -> int:
        return out_dim if out_dim else self.cfg.hidden_size

    def encode(self, ids, out_dim: int = 0) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros(self.out_width(out_dim), dtype=np.float32)
        err = C.create_string_buffer(512)
        if lib().fo_encode(self._h, ids.ctypes.data, len(ids), out_dim, out.ctypes.data, err, 512):
            raise OracleError(err.value.decode())
        return out

    def encode_batch(self, ids, cu, out_dim: int = 0, threads: Optional[int] = None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        cu = np.ascontiguousarray(cu, dtype=np.int32)
        n = len(cu) - 1
        out = np.zeros((n, self.out_width(out_dim)), dtype=np.float32)
        err = C.create_string_buffer(512)
        t = threads or os.cpu_count() or 1
        if lib().fo_encode_batch(self._h, ids.ctypes.data, cu.ctypes.data, n, out_dim,
                                 out.ctypes.data, t, err, 512):
            raise OracleError(err.value.decode())
        return out

    def q8_weight(self, layer: int, slot: int):
        """Requantised (int8 [n, k], scales [n]) of layer GEMM `slot`
        (0 qkv, 1 out, 2 fc1, 3 gate, 4 fc2)."""
        h, inter = self.cfg.hidden_size, self.cfg.intermediate_size
        nk = [(3 * h, h), (h, h), (inter, h), (inter, h), (h, inter)][slot]
        dp = lib().fo_q8_data(self._h, layer, slot)
        sp = lib().fo_q8_scale(self._h, layer, slot)
        if not dp:
            return None
        d = np.ctypeslib.as_array(C.cast(dp, C.POINTER(C.c_int8)), shape=(nk[0] * nk[1],))
        s = np.ctypeslib.as_array(C.cast(sp, C.POINTER(C.c_float)), shape=(nk[0],))
        return d.reshape(nk).copy(), s.copy()


# ---- kernel-level restatements ------------------------------------------------
def matmul_t(a, b, bias=None, avx2: bool = False) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    n = b.shape[0]
    out = np.zeros((m, n), dtype=np.float32)
    bias = None if bias is None else _f32(bias)
    fn = lib().fo_matmul_t_avx2 if avx2 else lib().fo_matmul_t
    fn(out.ctypes.data, a.ctypes.data, b.ctypes.data, m, n, k, _ptr(bias))
    return out


def quantize_rows_q8(x):
    x = _f32(x)
    rows, k = x.shape
    q = np.zeros((rows, k), dtype=np.int8)
    s = np.zeros(rows, dtype=np.float32)
    for r in range(rows):
        s[r] = lib().fo_quantize_row_q8(q[r].ctypes.data, x[r].ctypes.data, k)
    return q, s


def matmul_t_q8(a, qb, scales, bias=None) -> np.ndarray:
    a = _f32(a)
    qb = np.ascontiguousarray(qb, dtype=np.int8)
    scales = _f32(scales)
    m, k = a.shape
    n = qb.shape[0]
    out = np.zeros((m, n), dtype=np.float32)
    bias = None if bias is None else _f32(bias)
    lib().fo_matmul_t_q8(out.ctypes.data, a.ctypes.data, qb.ctypes.data, scales.ctypes.data,
                         m, n, k, _ptr(bias))
    return out


def layernorm_rows(x, w=None, b=None, eps=1e-12) -> np.ndarray:
    x = _f32(x).copy()
    rows, h = x.shape
    w = None if w is None else _f32(w)
    b = None if b is None else _f32(b)
    lib().fo_layernorm_rows(x.ctypes.data, rows, h, _ptr(w), _ptr(b), eps)
    return x


def softmax_scaled(row, scale: float) -> np.ndarray:
    r = _f32(row).copy()
    lib().fo_softmax_scaled(r.ctypes.data, len(r), scale)
    return r


def exp_f32(x: float) -> float:
    return lib().fo_exp(x)


def gelu_f32(x: float) -> float:
    return lib().fo_gelu(x)


def sigmoid_f32(x: float) -> float:
    return lib().fo_sigmoid(x)


def rope_tables(max_seq: int, head_dim: int, theta: float):
    half = head_dim // 2
    c = np.zeros((max_seq, half), dtype=np.float32)
    s = np.zeros((max_seq, half), dtype=np.float32)
    lib().fo_rope_tables(max_seq, head_dim, theta, c.ctypes.data, s.ctypes.data)
    return c, s


def attend_head(qkv, hd: int, head: int, rows: Optional[int] = None, rope=None,
                gemm: int = GEMM_GO) -> np.ndarray:
    """attendHead (model.go:646-701) for one head of one sequence: qkv is its
    [seq, 3h] float32 block; the first `rows` queries (default: all) attend
    over every key; rope = (cos, sin) tables [positions, hd/2] or None.
    Returns [rows, hd]."""
    qkv = _f32(qkv)
    seq, h = qkv.shape[0], qkv.shape[1] // 3
    rows = seq if rows is None else rows
    out = np.zeros((rows, hd), dtype=np.float32)
    rc, rs = (None, None) if rope is None else (_f32(rope[0]), _f32(rope[1]))
    if lib().fo_attend_head(qkv.ctypes.data, seq, rows, h, hd, head, _ptr(rc), _ptr(rs), gemm,
                            out.ctypes.data):
        raise OracleError("fo_attend_head: bad shape")
    return out


def has_avx2() -> bool:
    return bool(lib().fo_has_avx2())
