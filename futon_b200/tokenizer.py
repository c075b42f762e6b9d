"""Native WordPiece tokenizer over libfuton_cuda (include/futon_tokenizer.h).

Mirror of the reference's Tokenizer (native/tokenizer.go), same names,
argument meaning and errors:

  Tokenizer.from_file(vocab_path, cfg)      NewTokenizer
  Tokenizer(vocab_bytes, cfg)               the same from vocab.txt's bytes
  tok.encode(text, max_seq_len) -> [int]    Encode: [CLS] … [SEP], truncated
  tok.encode_batch(texts, max_seq_len)      Encode of every text on all host
                                            threads, packed as (ids, cu_seqlens)
                                            for Model.encode_packed / encode_batch
  tok.vocab_size(), tok.pad_id()            VocabSize, PadID

The work runs in C++ in the library (no Python fallback); it needs no GPU.
Errors raise FutonError with the reference's "tokenizer:" messages.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import os
from typing import List, Optional, Sequence, Tuple, Union

import numpy as np

from . import _lib
from ._lib import FutonError

Text = Union[str, bytes]


@dataclasses.dataclass
class TokenizerConfig:
    """TokenizerConfig (tokenizer.go:15-32): a pack config's "tokenizer"
    object. Empty fields take the defaults of applyDefaults (:34-55)."""

    do_lower_case: bool = False
    tokenize_chinese_chars: bool = False
    max_input_chars_per_word: int = 0
    cls_token: str = ""
    sep_token: str = ""
    unk_token: str = ""
    pad_token: str = ""
    mask_token: str = ""

    @classmethod
    def from_dict(cls, d: Optional[dict]) -> "TokenizerConfig":
        d = d or {}
        return cls(**{f.name: d[f.name] for f in dataclasses.fields(cls) if f.name in d})


def _as_bytes(t: Text) -> bytes:
    return t.encode("utf-8", "surrogatepass") if isinstance(t, str) else bytes(t)


def pack_texts(texts: Sequence[Text]) -> Tuple[bytes, np.ndarray]:
    """Concatenated UTF-8 bytes and int64 offsets [n+1] of texts. A list of
    str is joined once and encoded once (an ASCII str's length is its byte
    count; others are measured by encoding them)."""
    offsets = np.zeros(len(texts) + 1, dtype=np.int64)
    if not texts:
        return b"", offsets
    if all(isinstance(t, str) for t in texts):
        lens = [len(t) if t.isascii() else len(t.encode("utf-8", "surrogatepass"))
                for t in texts]
        data = "".join(texts).encode("utf-8", "surrogatepass")
    else:
        parts = [_as_bytes(t) for t in texts]
        lens = [len(p) for p in parts]
        data = b"".join(parts)
    np.cumsum(np.asarray(lens, dtype=np.int64), out=offsets[1:])
    return data, offsets


class Tokenizer:
    """native.Tokenizer backed by the library's C++ implementation."""

    def __init__(self, vocab: bytes, cfg: Optional[TokenizerConfig] = None):
        cfg = cfg or TokenizerConfig()
        self.cfg = cfg
        self._keep = [s.encode() if s else None for s in
                      (cfg.cls_token, cfg.sep_token, cfg.unk_token, cfg.pad_token, cfg.mask_token)]
        c = _lib.FutonTokenizerCfg(int(bool(cfg.do_lower_case)),
                                   int(bool(cfg.tokenize_chinese_chars)),
                                   int(cfg.max_input_chars_per_word), *self._keep)
        self._vocab = bytes(vocab)
        handle = C.c_void_p()
        _lib.call("futon_tokenizer_create", self._vocab, len(self._vocab), C.byref(c),
                  C.byref(handle))
        self._h = handle
        self._lib = _lib.lib()

    @classmethod
    def from_file(cls, vocab_path: os.PathLike, cfg: Optional[TokenizerConfig] = None
                  ) -> "Tokenizer":
        """NewTokenizer (tokenizer.go:90-136)."""
        try:
            with open(vocab_path, "rb") as f:
                data = f.read()
        except OSError as e:
            raise FutonError(_lib.FUTON_EINVAL, f"tokenizer: open vocab: {e}") from e
        return cls(data, cfg)

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            self._lib.futon_tokenizer_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def vocab_size(self) -> int:
        return int(self._lib.futon_tokenizer_vocab_size(self._h))

    def pad_id(self) -> int:
        return int(self._lib.futon_tokenizer_pad_id(self._h))

    def encode(self, text: Text, max_seq_len: int) -> List[int]:
        """Encode (tokenizer.go:143-184)."""
        b = _as_bytes(text)
        # As in encode_packed_bytes: ids ≤ bytes + 2 in practice, and a short
        # buffer comes back with the exact count, then the call is repeated.
        cap = min(max(2, max_seq_len), len(b) + 2)
        n = C.c_int(0)
        for _ in range(2):
            out = (C.c_int32 * cap)()
            try:
                _lib.call("futon_tokenizer_encode", self._h, b, len(b), int(max_seq_len), out,
                          cap, C.byref(n))
                return list(out[:n.value])
            except FutonError:
                if n.value <= cap:
                    raise
                cap = n.value
        raise FutonError(_lib.FUTON_EINVAL, "tokenizer: id count changed between calls")

    def encode_packed_bytes(self, data: bytes, offsets: np.ndarray, max_seq_len: int,
                            threads: int = 0) -> Tuple[np.ndarray, np.ndarray]:
        """encode_batch over texts already concatenated: text i is
        data[offsets[i]:offsets[i+1]]."""
        offsets = np.ascontiguousarray(offsets, dtype=np.int64)
        n = len(offsets) - 1
        if n < 0:
            raise FutonError(_lib.FUTON_EINVAL, "tokenizer: offsets must hold n+1 entries")
        if n > 0 and (offsets[0] < 0 or offsets[-1] > len(data)):
            raise FutonError(_lib.FUTON_EINVAL, "tokenizer: offsets outside the text buffer")
        cu = np.zeros(n + 1, dtype=np.int32)
        if n == 0:
            return np.zeros(0, dtype=np.int32), cu
        # Every id consumes at least one input byte besides [CLS]/[SEP]; a
        # short buffer is reported with the exact total in cu, then retried.
        lens = np.diff(offsets)
        cap = int(np.minimum(lens + 2, max(2, max_seq_len)).sum())
        for _ in range(2):
            ids = np.empty(cap, dtype=np.int32)
            try:
                _lib.call("futon_tokenizer_encode_batch", self._h, data, offsets.ctypes.data, n,
                          int(max_seq_len), int(threads), ids.ctypes.data, cap, cu.ctypes.data)
                return ids[:int(cu[-1])], cu
            except FutonError:
                if int(cu[-1]) <= cap:
                    raise
                cap = int(cu[-1])
        raise FutonError(_lib.FUTON_EINVAL, "tokenizer: batch size changed between calls")

    def encode_batch(self, texts: Sequence[Text], max_seq_len: int, threads: int = 0
                     ) -> Tuple[np.ndarray, np.ndarray]:
        """Encode of every text (threads = 0: all hardware threads), packed
        as (ids int32 [Σ L], cu_seqlens int32 [n+1]); equal to encode per
        text for every thread count."""
        data, offsets = pack_texts(texts)
        return self.encode_packed_bytes(data, offsets, max_seq_len, threads)
