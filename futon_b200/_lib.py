"""ctypes binding of libfuton_cuda.so (the C ABI in include/futon_cuda.h and
include/futon_tokenizer.h).

The library lives next to this file. There is no fallback: if it is missing
or fails to load, every entry point raises FutonLibraryError.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfuton_cuda.so"

FUTON_OK, FUTON_EINVAL, FUTON_ECUDA, FUTON_ECANCELED, FUTON_ENOMEM, FUTON_EDEVICE = range(6)
POS_ABSOLUTE, POS_ROPE = 0, 1
ACT_GELU, ACT_SWIGLU = 0, 1
POOL_CLS, POOL_MEAN = 0, 1
DTYPE_F32, DTYPE_F16 = 0, 1

# Every function the header declares (checked by the CPU test suite).
EXPORTED = (
    "futon_cuda_device_count", "futon_cuda_model_create", "futon_cuda_model_destroy",
    "futon_cuda_encode", "futon_cuda_encode_batch", "futon_cuda_encode_device",
    "futon_cuda_sync", "futon_cuda_launch_count", "futon_cuda_matmul_t",
    "futon_cuda_matmul_t_q8", "futon_cuda_quantize_rows_q8", "futon_cuda_profile",
    "futon_cuda_profile_read", "futon_cuda_profile_stage_count", "futon_cuda_profile_stage_name",
    "futon_cuda_matmul_t_q8_noalloc", "futon_cuda_selftest_wait_timeout", "futon_cuda_io_bytes",
    "futon_cuda_debug_cancel_after",
    "futon_tokenizer_create", "futon_tokenizer_destroy", "futon_tokenizer_vocab_size",
    "futon_tokenizer_pad_id", "futon_tokenizer_encode", "futon_tokenizer_encode_batch",
)

# Environment options the library reads when a model is created, with the
# values it accepts (any other value leaves the default, listed first).
RUNTIME_OPTIONS = {
    "FUTON_CUDA_ATTN": ("heads", "tc2"),
    "FUTON_CUDA_ATTN_SPLIT": ("1", "0"),
    "FUTON_CUDA_Q8_ATTN": ("exact", "split"),
    "FUTON_CUDA_GEMM_PAIR": ("0", "1"),
}


class FutonLibraryError(RuntimeError):
    """libfuton_cuda.so is missing or could not be loaded."""


class FutonError(RuntimeError):
    """An entry point returned a non-zero FUTON_E* code."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


class CanceledError(FutonError):
    """The cancel flag was raised (the reference returns context.Canceled)."""


class FutonCfg(C.Structure):
    _fields_ = [
        ("hidden_size", C.c_int32), ("num_layers", C.c_int32), ("num_heads", C.c_int32),
        ("intermediate_size", C.c_int32), ("vocab_size", C.c_int32),
        ("type_vocab_size", C.c_int32), ("max_seq_len", C.c_int32),
        ("max_trained_positions", C.c_int32), ("layer_norm_eps", C.c_double),
        ("position_encoding", C.c_int32), ("rope_theta", C.c_double),
        ("activation", C.c_int32), ("pooling", C.c_int32), ("normalize", C.c_int32),
        ("matryoshka", C.c_int32), ("matryoshka_layernorm", C.c_int32),
    ]


class FutonTokenizerCfg(C.Structure):
    _fields_ = [
        ("do_lower_case", C.c_int32), ("tokenize_chinese_chars", C.c_int32),
        ("max_input_chars_per_word", C.c_int32), ("cls_token", C.c_char_p),
        ("sep_token", C.c_char_p), ("unk_token", C.c_char_p), ("pad_token", C.c_char_p),
        ("mask_token", C.c_char_p),
    ]


class FutonTensor(C.Structure):
    _fields_ = [
        ("name", C.c_char_p), ("dtype", C.c_int32), ("ndim", C.c_int32),
        ("shape", C.c_int64 * 4), ("data", C.c_void_p),
    ]


_lock = threading.Lock()
_lib = None


def lib() -> C.CDLL:
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise FutonLibraryError(
                f"{LIB_PATH} not found: build it with `python -m futon_b200.build` "
                "(there is no CPU fallback)")
        try:
            L = C.CDLL(str(LIB_PATH))
        except OSError as e:
            raise FutonLibraryError(f"failed to load {LIB_PATH}: {e}") from e
        vp, ip, i32p = C.c_void_p, C.c_int, C.POINTER(C.c_int32)
        cp, sz = C.c_char_p, C.c_size_t
        L.futon_cuda_device_count.restype = ip
        L.futon_cuda_device_count.argtypes = []
        L.futon_cuda_model_create.restype = ip
        L.futon_cuda_model_create.argtypes = [C.POINTER(FutonCfg), C.POINTER(FutonTensor), ip,
                                              C.POINTER(C.c_int), ip, ip, C.POINTER(vp), cp, sz]
        L.futon_cuda_model_destroy.restype = None
        L.futon_cuda_model_destroy.argtypes = [vp]
        L.futon_cuda_encode.restype = ip
        L.futon_cuda_encode.argtypes = [vp, ip, vp, vp, ip, ip, vp, vp, cp, sz]
        L.futon_cuda_encode_batch.restype = ip
        L.futon_cuda_encode_batch.argtypes = [vp, vp, vp, ip, ip, vp, vp, cp, sz]
        L.futon_cuda_encode_device.restype = ip
        L.futon_cuda_encode_device.argtypes = [vp, ip, vp, vp, ip, ip, vp, vp, cp, sz]
        L.futon_cuda_sync.restype = ip
        L.futon_cuda_sync.argtypes = [vp, ip, vp, cp, sz]
        L.futon_cuda_launch_count.restype = C.c_longlong
        L.futon_cuda_launch_count.argtypes = [vp, ip]
        L.futon_cuda_io_bytes.restype = ip
        L.futon_cuda_io_bytes.argtypes = [vp, ip, C.POINTER(C.c_longlong), C.POINTER(C.c_longlong),
                                          cp, sz]
        L.futon_cuda_profile.restype = ip
        L.futon_cuda_profile.argtypes = [vp, ip, ip, cp, sz]
        L.futon_cuda_profile_read.restype = ip
        L.futon_cuda_profile_read.argtypes = [vp, ip, ip, C.POINTER(C.c_double),
                                              C.POINTER(C.c_longlong), C.POINTER(C.c_double),
                                              C.POINTER(C.c_double), cp, sz]
        L.futon_cuda_profile_stage_count.restype = ip
        L.futon_cuda_profile_stage_count.argtypes = []
        L.futon_cuda_profile_stage_name.restype = C.c_char_p
        L.futon_cuda_profile_stage_name.argtypes = [ip]
        L.futon_cuda_matmul_t.restype = ip
        L.futon_cuda_matmul_t.argtypes = [ip, vp, vp, vp, ip, ip, ip, vp, vp, cp, sz]
        L.futon_cuda_matmul_t_q8.restype = ip
        L.futon_cuda_matmul_t_q8.argtypes = [ip, vp, vp, vp, vp, ip, ip, ip, vp, vp, cp, sz]
        L.futon_cuda_matmul_t_q8_noalloc.restype = ip
        L.futon_cuda_matmul_t_q8_noalloc.argtypes = [ip, vp, vp, vp, vp, ip, ip, ip, vp, vp, cp, sz]
        L.futon_cuda_quantize_rows_q8.restype = ip
        L.futon_cuda_quantize_rows_q8.argtypes = [ip, vp, vp, vp, ip, ip, vp, cp, sz]
        L.futon_cuda_selftest_wait_timeout.restype = ip
        L.futon_cuda_selftest_wait_timeout.argtypes = [ip, cp, sz]
        L.futon_cuda_debug_cancel_after.restype = None
        L.futon_cuda_debug_cancel_after.argtypes = [C.c_longlong]
        L.futon_tokenizer_create.restype = ip
        L.futon_tokenizer_create.argtypes = [vp, sz, C.POINTER(FutonTokenizerCfg), C.POINTER(vp),
                                             cp, sz]
        L.futon_tokenizer_destroy.restype = None
        L.futon_tokenizer_destroy.argtypes = [vp]
        L.futon_tokenizer_vocab_size.restype = ip
        L.futon_tokenizer_vocab_size.argtypes = [vp]
        L.futon_tokenizer_pad_id.restype = ip
        L.futon_tokenizer_pad_id.argtypes = [vp]
        L.futon_tokenizer_encode.restype = ip
        L.futon_tokenizer_encode.argtypes = [vp, vp, sz, ip, vp, ip, C.POINTER(C.c_int), cp, sz]
        L.futon_tokenizer_encode_batch.restype = ip
        L.futon_tokenizer_encode_batch.argtypes = [vp, vp, vp, ip, ip, ip, vp, C.c_int64, vp, cp,
                                                   sz]
        _lib = L
        return L


def call(fn_name: str, *args) -> None:
    """Calls an int-returning entry point with a trailing (err, errlen) pair
    and raises FutonError / CanceledError on failure."""
    buf = C.create_string_buffer(1024)
    rc = getattr(lib(), fn_name)(*args, buf, C.sizeof(buf))
    if rc != FUTON_OK:
        msg = buf.value.decode("utf-8", "replace") or f"{fn_name} failed with code {rc}"
        if rc == FUTON_ECANCELED:
            raise CanceledError(rc, msg)
        raise FutonError(rc, msg)


def device_count() -> int:
    return int(lib().futon_cuda_device_count())


def env_flag(name: str) -> bool:
    return os.environ.get(name, "") == "1"
