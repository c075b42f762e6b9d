"""Python mirror of futon's native Provider over libfuton_cuda.

Same names, argument meaning and error behaviour as the Go surface
(native/provider.go:36-290, native/model.go:112-457):

  Model.load(pack_dir)            LoadModel: manifest + config + tensors,
                                  uploaded once per device (one replica each)
  Model.encode_tokens(ids, dim)   EncodeTokens for one sequence
  Model.encode_packed(ids, cu)    many sequences in one call (packed, no padding)
  Provider(Options(...))          New: pack load, tokenizer from vocab.txt,
                                  Dimensions validation
  Provider.embed / embed_batch    Embed / EmbedBatch: text → native tokenizer
                                  (tokenizer.py) → forward (embed_texts)
  Provider.embed_ids / embed_batch_ids   the same for pre-tokenised input
  Provider.dimensions / model_name / is_available / close

Errors carry the reference's "native:" messages; a raised cancel flag
surfaces as CanceledError. There is no CPU path: every forward runs the
CUDA kernels in libfuton_cuda.so.
"""
from __future__ import annotations

import contextlib
import ctypes as C
import dataclasses
import threading
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import FutonError
from .pack import (ACT_SWIGLU, POOL_MEAN, POS_ROPE, PackConfig, PackError, load_pack)
from .tokenizer import Text, Tokenizer, TokenizerConfig

NATIVE_MODEL_NAME_PREFIX = "native/"
ENV_NATIVE_Q8 = "FUTON_NATIVE_Q8"


class CancelFlag:
    """A cancellation flag the library polls between micro-batches and layers
    (the GPU counterpart of the reference's context checkpoints)."""

    def __init__(self) -> None:
        self._v = C.c_int(0)

    def cancel(self) -> None:
        self._v.value = 1

    def is_set(self) -> bool:
        return self._v.value != 0

    @property
    def ptr(self) -> int:
        return C.addressof(self._v)


def _cfg_struct(cfg: PackConfig) -> _lib.FutonCfg:
    c = _lib.FutonCfg()
    c.hidden_size = cfg.hidden_size
    c.num_layers = cfg.num_layers
    c.num_heads = cfg.num_heads
    c.intermediate_size = cfg.intermediate_size
    c.vocab_size = cfg.vocab_size
    c.type_vocab_size = cfg.type_vocab_size
    c.max_seq_len = cfg.max_seq_len
    c.max_trained_positions = cfg.max_trained_positions
    c.layer_norm_eps = cfg.layer_norm_eps
    c.position_encoding = _lib.POS_ROPE if cfg.position_encoding == POS_ROPE else _lib.POS_ABSOLUTE
    c.rope_theta = cfg.rope_theta
    c.activation = _lib.ACT_SWIGLU if cfg.activation == ACT_SWIGLU else _lib.ACT_GELU
    c.pooling = _lib.POOL_MEAN if cfg.pooling == POOL_MEAN else _lib.POOL_CLS
    c.normalize = 1 if cfg.normalize else 0
    c.matryoshka = 1 if cfg.matryoshka is not None else 0
    c.matryoshka_layernorm = 1 if (cfg.matryoshka is not None and cfg.matryoshka.layernorm) else 0
    return c


# Text bytes of the first chunk of a pipelined embed_batch (~1M tokens of
# English text: two full micro-batches of the forward).
FIRST_CHUNK_BYTES = 8 << 20


def text_chunks(texts: Sequence[Text], first_bytes: int = FIRST_CHUNK_BYTES) -> List[tuple]:
    """[lo, hi) text ranges of a pipelined embed_batch: the first holds about
    first_bytes of text, each next one about twice the previous, the last
    takes the rest (a batch under 2 × first_bytes stays whole)."""
    sizes = np.fromiter((len(t) for t in texts), dtype=np.int64, count=len(texts))
    csum = np.cumsum(sizes)
    total = int(csum[-1]) if len(texts) else 0
    chunks, lo, want, done = [], 0, first_bytes, 0
    while lo < len(texts):
        if total - done < 2 * want:
            chunks.append((lo, len(texts)))
            break
        hi = int(np.searchsorted(csum, done + want, side="left")) + 1
        hi = min(max(hi, lo + 1), len(texts))
        chunks.append((lo, hi))
        done = int(csum[hi - 1])
        lo, want = hi, 2 * want
    return chunks


def embed_texts(model: "Model", tokenizer: Tokenizer, texts: Sequence[Text], out_dim: int = 0,
                threads: int = 0, cancel: Optional[CancelFlag] = None) -> np.ndarray:
    """Texts → [n, out_dim or hidden] vectors over every device of `model`.
    Texts are tokenised on `threads` host threads (0 = all), truncated to
    the model's EffectiveMaxSeqLen, and encoded by packed forwards sharded
    across the GPUs. A large batch goes in chunks that double in size
    (text_chunks): while the GPUs encode chunk k, a host thread tokenises
    chunk k+1 (the library call releases the GIL), so only the first
    chunk's tokenisation is exposed. Results do not depend on the chunking."""
    n = len(texts)
    out = np.empty((n, model.out_width(out_dim)), dtype=np.float32)
    if n == 0:
        return out
    max_len = model.effective_max_seq_len()
    chunks = text_chunks(texts, FIRST_CHUNK_BYTES)

    def tokenize(k):
        lo, hi = chunks[k]
        return tokenizer.encode_batch(texts[lo:hi], max_len, threads)

    if len(chunks) == 1:
        ids, cu = tokenize(0)
        return model.encode_batch(ids, cu, out_dim, cancel=cancel, out=out)
    with ThreadPoolExecutor(max_workers=1) as ex:
        nxt = ex.submit(tokenize, 0)
        for k, (lo, hi) in enumerate(chunks):
            ids, cu = nxt.result()
            if k + 1 < len(chunks):
                nxt = ex.submit(tokenize, k + 1)
            model.encode_batch(ids, cu, out_dim, cancel=cancel, out=out[lo:hi])
    return out


def pack_ids(seqs: Sequence[Sequence[int]]) -> tuple:
    """Packs id sequences into (ids int32 [Σ L], cu_seqlens int32 [n+1])."""
    lens = np.fromiter((len(s) for s in seqs), dtype=np.int64, count=len(seqs))
    cu = np.zeros(len(seqs) + 1, dtype=np.int32)
    np.cumsum(lens, out=cu[1:])
    ids = (np.concatenate([np.asarray(s, dtype=np.int32) for s in seqs])
           if len(seqs) else np.zeros(0, dtype=np.int32))
    return np.ascontiguousarray(ids, dtype=np.int32), cu


class Model:
    """A pack uploaded to one or more GPUs (LoadModel + newModel)."""

    def __init__(self, cfg: PackConfig, tensors: Dict[str, np.ndarray],
                 devices: Optional[Sequence[int]] = None, q8: Optional[bool] = None):
        cfg.validate()
        if q8 is None:
            q8 = _lib.env_flag(ENV_NATIVE_Q8)
        ndev = _lib.device_count()
        if devices is None:
            devices = list(range(ndev))
        devices = list(devices)
        if not devices:
            raise FutonError(_lib.FUTON_EINVAL, "native: no CUDA device visible")
        self.cfg = cfg
        self.q8 = bool(q8)
        self.devices = devices
        keep = []
        arr = (_lib.FutonTensor * max(1, len(tensors)))()
        for i, name in enumerate(sorted(tensors)):
            t = tensors[name]
            if t.dtype == np.float16:
                dt = _lib.DTYPE_F16
            else:
                t = np.ascontiguousarray(t, dtype=np.float32)
                dt = _lib.DTYPE_F32
            t = np.ascontiguousarray(t)
            keep.append(t)
            if t.ndim < 1 or t.ndim > 4:
                raise PackError(f"pack {cfg.model_id}: tensor {name!r} rank {t.ndim}")
            arr[i].name = name.encode()
            arr[i].dtype = dt
            arr[i].ndim = t.ndim
            for k, s in enumerate(t.shape):
                arr[i].shape[k] = s
            arr[i].data = t.ctypes.data
        devs = (C.c_int * len(devices))(*devices)
        handle = C.c_void_p()
        cs = _cfg_struct(cfg)
        _lib.call("futon_cuda_model_create", C.byref(cs), arr, len(tensors), devs, len(devices),
                  1 if self.q8 else 0, C.byref(handle))
        self._init_handle(handle)

    def _init_handle(self, handle: C.c_void_p) -> None:
        self._h = handle
        self._closed = False
        self._cv = threading.Condition()
        self._inflight = 0

    @classmethod
    def load(cls, pack_dir, devices=None, q8=None) -> "Model":
        p = load_pack(pack_dir, keep_f16=True)
        return cls(p.cfg, p.tensors, devices=devices, q8=q8)

    # -- lifecycle --------------------------------------------------------
    def close(self) -> None:
        """Refuses new calls, waits for the calls in flight on other threads
        (like Provider.Close, provider.go:274-281, which lets in-flight
        forwards finish), then releases every device buffer."""
        with self._cv:
            self._closed = True
            while self._inflight:
                self._cv.wait()
            if self._h:
                _lib.lib().futon_cuda_model_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> C.c_void_p:
        if self._closed:
            raise FutonError(_lib.FUTON_EINVAL, "native: model is closed")
        return self._h

    @contextlib.contextmanager
    def _call(self):
        """The native handle for one call; close() waits until it returns."""
        with self._cv:
            if self._closed:
                raise FutonError(_lib.FUTON_EINVAL, "native: model is closed")
            self._inflight += 1
            h = self._h
        try:
            yield h
        finally:
            with self._cv:
                self._inflight -= 1
                if not self._inflight:
                    self._cv.notify_all()

    def effective_max_seq_len(self) -> int:
        return self.cfg.effective_max_seq_len()

    def out_width(self, out_dim: int) -> int:
        return out_dim if out_dim else self.cfg.hidden_size

    # -- forward ----------------------------------------------------------
    def encode_packed(self, ids: np.ndarray, cu_seqlens: np.ndarray, out_dim: int = 0,
                      device: int = 0, cancel: Optional[CancelFlag] = None,
                      out: Optional[np.ndarray] = None) -> np.ndarray:
        """[nseq, dim] vectors for packed sequences on device index `device`,
        written to `out` when given (a C-contiguous float32 [nseq, dim] host
        array, e.g. rows of a caller's index-aligned result buffer)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        nseq = len(cu) - 1
        shape = (max(nseq, 0), self.out_width(out_dim))
        if out is None:
            out = np.empty(shape, dtype=np.float32)
        elif out.shape != shape or out.dtype != np.float32 or not out.flags.c_contiguous:
            raise FutonError(_lib.FUTON_EINVAL,
                             f"native: out must be C-contiguous float32 {shape}, got "
                             f"{out.dtype} {out.shape}")
        with self._call() as h:
            _lib.call("futon_cuda_encode", h, device, ids.ctypes.data, cu.ctypes.data, nseq,
                      out_dim, out.ctypes.data, cancel.ptr if cancel else None)
        return out

    def encode_batch(self, ids: np.ndarray, cu_seqlens: np.ndarray, out_dim: int = 0,
                     cancel: Optional[CancelFlag] = None,
                     out: Optional[np.ndarray] = None) -> np.ndarray:
        """Data-parallel over every device of the model (EmbedBatch's engine),
        written to `out` when given (as in encode_packed)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        nseq = len(cu) - 1
        shape = (max(nseq, 0), self.out_width(out_dim))
        if out is None:
            out = np.empty(shape, dtype=np.float32)
        elif out.shape != shape or out.dtype != np.float32 or not out.flags.c_contiguous:
            raise FutonError(_lib.FUTON_EINVAL,
                             f"native: out must be C-contiguous float32 {shape}, got "
                             f"{out.dtype} {out.shape}")
        with self._call() as h:
            _lib.call("futon_cuda_encode_batch", h, ids.ctypes.data, cu.ctypes.data, nseq,
                      out_dim, out.ctypes.data, cancel.ptr if cancel else None)
        return out

    def encode_tokens(self, ids: Sequence[int], out_dim: int = 0, device: int = 0,
                      cancel: Optional[CancelFlag] = None) -> np.ndarray:
        """EncodeTokens (model.go:335-457) for one id sequence."""
        ids = np.asarray(ids, dtype=np.int64)
        if ids.size == 0:
            raise FutonError(_lib.FUTON_EINVAL, "native: empty token sequence")
        if ids.min() < np.iinfo(np.int32).min or ids.max() > np.iinfo(np.int32).max:
            raise FutonError(_lib.FUTON_EINVAL, "native: token id outside vocab")
        cu = np.array([0, ids.size], dtype=np.int32)
        return self.encode_packed(ids.astype(np.int32), cu, out_dim, device, cancel)[0]

    def encode_device(self, d_ids: int, cu_seqlens: np.ndarray, out_dim: int, d_out: int,
                      device: int = 0, stream: Optional[int] = None) -> None:
        """Queues a forward over ids already in HBM (returns without waiting)."""
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        with self._call() as h:
            _lib.call("futon_cuda_encode_device", h, device, C.c_void_p(d_ids),
                      cu.ctypes.data, len(cu) - 1, out_dim, C.c_void_p(d_out),
                      C.c_void_p(stream) if stream else None)

    def sync(self, device: int = 0, stream: Optional[int] = None) -> None:
        with self._call() as h:
            _lib.call("futon_cuda_sync", h, device, C.c_void_p(stream) if stream else None)

    def io_bytes(self, device: int = 0) -> tuple:
        """(host→device, device→host) bytes the calls on `device` copied since create."""
        h2d, d2h = C.c_longlong(), C.c_longlong()
        with self._call() as h:
            _lib.call("futon_cuda_io_bytes", h, device, C.byref(h2d), C.byref(d2h))
        return int(h2d.value), int(d2h.value)

    def launch_count(self, device: int = 0) -> int:
        with self._call() as h:
            return int(_lib.lib().futon_cuda_launch_count(h, device))

    def profile(self, enable: bool, device: int = 0) -> None:
        """Resets the per-stage profiler and turns it on or off."""
        with self._call() as h:
            _lib.call("futon_cuda_profile", h, device, 1 if enable else 0)

    def profile_read(self, device: int = 0) -> Dict[str, dict]:
        """{stage: {ms, launches, flops, bytes}} accumulated since profile(True)."""
        L = _lib.lib()
        out = {}
        with self._call() as h:
            for st in range(L.futon_cuda_profile_stage_count()):
                ms, n, fl, by = C.c_double(), C.c_longlong(), C.c_double(), C.c_double()
                _lib.call("futon_cuda_profile_read", h, device, st, C.byref(ms), C.byref(n),
                          C.byref(fl), C.byref(by))
                if n.value:
                    out[L.futon_cuda_profile_stage_name(st).decode()] = {
                        "ms": ms.value, "launches": n.value, "flops": fl.value, "bytes": by.value}
        return out


@dataclasses.dataclass
class Options:
    """native.Options (provider.go:55-65) plus the GPU selection."""

    pack_dir: str = ""
    dimensions: int = 0
    devices: Optional[List[int]] = None  # None = every visible GPU
    q8: Optional[bool] = None            # None = FUTON_NATIVE_Q8 == "1"
    threads: int = 0                     # host threads for tokenising a batch; 0 = all


class Provider:
    """native.Provider over the B200 engine (provider.go:36-290)."""

    def __init__(self, opts: Options):
        if not opts.pack_dir:
            raise FutonError(_lib.FUTON_EINVAL,
                             "native: PackDir is required (no downloading in this phase)")
        self.model = Model.load(opts.pack_dir, devices=opts.devices, q8=opts.q8)
        cfg = self.model.cfg
        try:
            self.tokenizer = Tokenizer.from_file(Path(opts.pack_dir) / "vocab.txt",
                                                 TokenizerConfig.from_dict(cfg.tokenizer))
        except FutonError:
            self.model.close()
            raise
        if self.tokenizer.vocab_size() > cfg.vocab_size:
            self.model.close()
            raise FutonError(_lib.FUTON_EINVAL,
                             f"native: vocab.txt has {self.tokenizer.vocab_size()} entries but "
                             f"pack declares vocab_size {cfg.vocab_size}")
        self._threads = opts.threads
        dims = opts.dimensions or cfg.hidden_size
        if dims != cfg.hidden_size:
            if cfg.matryoshka is None:
                self.model.close()
                raise FutonError(_lib.FUTON_EINVAL, f"native: pack {cfg.model_id} does not "
                                 f"support truncation to {dims} dimensions")
            if dims < 1 or dims > cfg.hidden_size:
                self.model.close()
                raise FutonError(_lib.FUTON_EINVAL,
                                 f"native: dimensions {dims} outside [1,{cfg.hidden_size}]")
        self._dims = dims
        self._mu = threading.Lock()
        self._closed = False

    def _check_open(self) -> None:
        with self._mu:
            if self._closed:
                raise FutonError(_lib.FUTON_EINVAL, "native: provider is closed")

    def embed(self, text: Text, cancel: Optional[CancelFlag] = None) -> np.ndarray:
        """Embed (provider.go:111-121): tokenise with the pack's vocab,
        truncated to EffectiveMaxSeqLen, then one forward."""
        self._check_open()
        ids = self.tokenizer.encode(text, self.model.effective_max_seq_len())
        return self.model.encode_tokens(ids, self._dims, cancel=cancel)

    def embed_batch(self, texts: Sequence[Text],
                    cancel: Optional[CancelFlag] = None) -> np.ndarray:
        """EmbedBatch (provider.go:152-202): index-aligned [n, dims] vectors,
        bit-identical to embed per text (embed_texts)."""
        self._check_open()
        return embed_texts(self.model, self.tokenizer, texts, self._dims, self._threads, cancel)

    def embed_ids(self, ids: Sequence[int], cancel: Optional[CancelFlag] = None) -> np.ndarray:
        """Embed for pre-tokenised input (provider.go:115-121)."""
        self._check_open()
        return self.model.encode_tokens(ids, self._dims, cancel=cancel)

    def embed_batch_ids(self, batch: Sequence[Sequence[int]],
                        cancel: Optional[CancelFlag] = None) -> np.ndarray:
        """EmbedBatch (provider.go:152-202): index-aligned [n, dims] vectors,
        sharded across every GPU; the first error fails the batch."""
        self._check_open()
        if len(batch) == 0:
            return np.zeros((0, self._dims), dtype=np.float32)
        for i, s in enumerate(batch):
            if len(s) == 0:
                raise FutonError(_lib.FUTON_EINVAL,
                                 f"native: batch item {i}: native: empty token sequence")
        ids, cu = pack_ids(batch)
        return self.model.encode_batch(ids, cu, self._dims, cancel=cancel)

    def dimensions(self) -> int:
        return self._dims

    def model_name(self) -> str:
        """Engine-qualified pack id (provider.go:261-264)."""
        return NATIVE_MODEL_NAME_PREFIX + self.model.cfg.model_id

    def is_available(self) -> bool:
        with self._mu:
            return not self._closed

    def close(self) -> None:
        with self._mu:
            if self._closed:
                return
            self._closed = True
        self.model.close()
        self.tokenizer.close()


def new(opts: Options) -> Provider:
    """native.New."""
    return Provider(opts)
