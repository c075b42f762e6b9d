"""ctypes bridge to libtokport.so, the compiled port of the reference tokenizer
in the reference's own structure (tokenizer_port.cpp) — TEST INFRASTRUCTURE
ONLY: bench.py times it as the text path's CPU baseline, and the tests check
its ids against the reference's fixtures and the library's tokenizer."""
from __future__ import annotations

import ctypes as C
from pathlib import Path
from typing import List, Tuple

import numpy as np

from . import oracle

LIB = Path(__file__).resolve().parent / "libtokport.so"
_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        oracle.build()
        L = C.CDLL(str(LIB))
        L.tp_create.restype = C.c_void_p
        L.tp_create.argtypes = [C.c_char_p, C.c_size_t, C.c_int, C.c_int]
        L.tp_destroy.restype = None
        L.tp_destroy.argtypes = [C.c_void_p]
        L.tp_encode_batch.restype = C.c_longlong
        L.tp_encode_batch.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_int, C.c_int,
                                      C.c_int, C.c_void_p, C.c_longlong, C.c_void_p]
        _lib = L
    return _lib


class TokenizerPort:
    """NewTokenizer + Encode with the default special tokens."""

    def __init__(self, vocab: bytes, do_lower_case: bool = True,
                 tokenize_chinese_chars: bool = True):
        self._vocab = bytes(vocab)
        self._h = lib().tp_create(self._vocab, len(self._vocab), int(do_lower_case),
                                  int(tokenize_chinese_chars))
        if not self._h:
            raise ValueError("tokenizer port: empty vocab or a special token missing")

    def __del__(self):
        if getattr(self, "_h", None):
            lib().tp_destroy(self._h)
            self._h = None

    def encode_packed_bytes(self, data: bytes, offsets: np.ndarray, max_seq_len: int,
                            threads: int = 1) -> Tuple[np.ndarray, np.ndarray]:
        offsets = np.ascontiguousarray(offsets, dtype=np.int64)
        n = len(offsets) - 1
        cu = np.zeros(n + 1, dtype=np.int32)
        cap = int(n * max(2, max_seq_len))
        ids = np.empty(max(cap, 1), dtype=np.int32)
        total = lib().tp_encode_batch(self._h, data, offsets.ctypes.data, n, int(max_seq_len),
                                      int(threads), ids.ctypes.data, cap, cu.ctypes.data)
        if total < 0:
            raise ValueError("tokenizer port: ids buffer too small")
        return ids[:total], cu

    def encode(self, text, max_seq_len: int) -> List[int]:
        b = text.encode("utf-8", "surrogatepass") if isinstance(text, str) else bytes(text)
        ids, _ = self.encode_packed_bytes(b, np.array([0, len(b)], np.int64), max_seq_len)
        return ids.tolist()
