"""The C-ABI library loads and exports every declared entry point; errors
come back as codes and messages, never crashes (no GPU needed)."""
from __future__ import annotations

import ctypes as C
import re

import numpy as np
import pytest

from conftest import GOLDEN, ROOT
from futon_b200 import FutonError, Model, _lib
from futon_b200.pack import load_pack


def declared(header) -> set:
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return set(re.findall(r"\b((?:futon|fo)_\w+)\s*\(", text))


def test_header_symbols_exported():
    headers = sorted((ROOT / "include").glob("*.h"))
    assert [h.name for h in headers] == ["futon_cuda.h", "futon_tokenizer.h"]
    names = set().union(*(declared(h) for h in headers))
    assert names == set(_lib.EXPORTED), names ^ set(_lib.EXPORTED)
    lib = C.CDLL(str(_lib.LIB_PATH))
    for n in names:
        assert hasattr(lib, n), n


def test_oracle_header_symbols_exported():
    from oracle import oracle as O
    names = declared(ROOT / "oracle" / "futon_oracle.h")
    lib = C.CDLL(str(O.build()))
    for n in names:
        assert hasattr(lib, n), n


def test_device_count_is_int():
    assert isinstance(_lib.device_count(), int)


def test_stage_names():
    L = _lib.lib()
    n = L.futon_cuda_profile_stage_count()
    names = [L.futon_cuda_profile_stage_name(i).decode() for i in range(n)]
    assert "gemm_fc1" in names and "attention" in names
    assert L.futon_cuda_profile_stage_name(n) == b""


def test_create_rejects_without_crashing():
    """Bad configurations return FUTON_EINVAL with a message (no GPU needed:
    validation runs before any device work)."""
    p = load_pack(GOLDEN / "toy-absolute-gelu")
    cfg = _lib.FutonCfg()
    handle = C.c_void_p()
    devs = (C.c_int * 1)(0)
    with pytest.raises(FutonError, match="non-positive"):
        _lib.call("futon_cuda_model_create", C.byref(cfg), None, 0, devs, 1, 0, C.byref(handle))
    if _lib.device_count() == 0:
        with pytest.raises(FutonError):
            Model(p.cfg, p.tensors, devices=[0])


def test_null_model_calls_return_errors():
    ids = np.array([2, 3], np.int32)
    cu = np.array([0, 2], np.int32)
    out = np.zeros((1, 32), np.float32)
    with pytest.raises(FutonError, match="null model"):
        _lib.call("futon_cuda_encode", None, 0, ids.ctypes.data, cu.ctypes.data, 1, 0,
                  out.ctypes.data, None)
    with pytest.raises(FutonError, match="null model"):
        _lib.call("futon_cuda_sync", None, 0, None)
    assert _lib.lib().futon_cuda_launch_count(None, 0) == -1
    h2d, d2h = C.c_longlong(), C.c_longlong()
    with pytest.raises(FutonError, match="bad model"):
        _lib.call("futon_cuda_io_bytes", None, 0, C.byref(h2d), C.byref(d2h))
    with pytest.raises(FutonError, match="null model"):
        _lib.call("futon_cuda_encode_device", None, 0, None, cu.ctypes.data, 1, 0, None, None)
    with pytest.raises(FutonError, match="null model"):
        _lib.call("futon_cuda_encode_batch", None, ids.ctypes.data, cu.ctypes.data, 1, 0,
                  out.ctypes.data, None)


@pytest.mark.parametrize("call", [
    ("futon_cuda_matmul_t", 0, None, None, None, 4, 4, 8, None, None),
    ("futon_cuda_matmul_t_q8", 0, None, None, None, None, 4, 4, 16, None, None),
    ("futon_cuda_matmul_t_q8_noalloc", 0, None, None, None, None, 4, 4, 16, None, None),
    ("futon_cuda_quantize_rows_q8", 0, None, None, None, 4, 16, None),
])
def test_kernel_seams_refuse_null_buffers(call):
    """Well-formed shapes with null buffers are refused before any device work."""
    with pytest.raises(FutonError, match="null buffer"):
        _lib.call(*call)


def test_kernel_seams_accept_empty_shapes():
    """m = 0 (or rows = 0) is a no-op that returns success without a device."""
    _lib.call("futon_cuda_matmul_t", 0, None, None, None, 0, 4, 8, None, None)
    _lib.call("futon_cuda_matmul_t_q8", 0, None, None, None, None, 0, 4, 16, None, None)
    _lib.call("futon_cuda_quantize_rows_q8", 0, None, None, None, 0, 16, None)


def test_runtime_options_match_library():
    """Every environment variable the library reads is in the package's
    RUNTIME_OPTIONS table, and every non-default value listed there is one
    the library compares against."""
    src = (ROOT / "futon_b200" / "csrc" / "futon_cuda.cu").read_text()
    names = set(re.findall(r'getenv\("(FUTON_\w+)"\)', src))
    assert names, "no environment options found"
    assert names == set(_lib.RUNTIME_OPTIONS), names ^ set(_lib.RUNTIME_OPTIONS)
    for n, values in _lib.RUNTIME_OPTIONS.items():
        for v in values[1:]:
            assert f'"{v}"' in src, f"{n}={v} is listed but not accepted"


def test_entry_points_forward_their_arguments():
    """Every C entry point reaches its body with its own arguments and
    returns that body's code and message through the exception guard at the
    ABI (invalid arguments, rejected before any device work, so no GPU is
    needed)."""
    E = _lib.FUTON_EINVAL
    d = C.c_double()
    ll = C.c_longlong()
    cases = [
        ("futon_cuda_encode", (None, 0, None, None, 0, 0, None, None), "null model"),
        ("futon_cuda_encode_batch", (None, None, None, 0, 0, None, None), "null model"),
        ("futon_cuda_encode_device", (None, 0, None, None, 0, 0, None, None), "null model"),
        ("futon_cuda_sync", (None, 0, None), "null model"),
        ("futon_cuda_io_bytes", (None, 0, C.byref(ll), C.byref(ll)), "bad model or device"),
        ("futon_cuda_profile", (None, 0, 1), "bad model or device"),
        ("futon_cuda_profile_read", (None, 0, 0, C.byref(d), C.byref(ll), C.byref(d), C.byref(d)),
         "bad model or device"),
        ("futon_cuda_matmul_t", (0, None, None, None, 4, 8, 7, None, None), r"m=4 n=8 k=7"),
        ("futon_cuda_matmul_t_q8", (0, None, None, None, None, 4, 8, 24, None, None),
         r"m=4 n=8 k=24"),
        ("futon_cuda_quantize_rows_q8", (0, None, None, None, 3, 6, None), r"rows=3 k=6"),
        ("futon_cuda_selftest_wait_timeout", (-1,), "bad device -1"),
    ]
    for fn, args, msg in cases:
        with pytest.raises(FutonError, match=msg) as ei:
            _lib.call(fn, *args)
        assert ei.value.code == E, fn


def test_headers_build_as_c_and_the_library_runs_from_c(tmp_path):
    """cgo compiles the headers as C: a pedantic C99 program includes both,
    links libfuton_cuda and tokenises the reference's fixture texts through
    the batch entry point (tests/host/abi_consumer.c), giving the fixture ids."""
    import json
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    exe = tmp_path / "abi_consumer"
    lib_dir = _lib.LIB_PATH.parent
    r = subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic",
                        "-I", str(ROOT / "include"), str(ROOT / "tests" / "host" / "abi_consumer.c"),
                        "-L", str(lib_dir), "-lfuton_cuda", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    tokdir = ROOT / "tests" / "golden" / "tokenizer"
    fx = json.loads((tokdir / "tokenizer_fixtures.json").read_text())
    cases = [c for c in fx["models"]["bge-small-en-v1.5"]["cases"] if "\x00" not in c["text"]]
    for max_len, key in ((512, "ids"), (16, "ids_max16")):
        r = subprocess.run([str(exe), str(tokdir / "vocab_bert_uncased.txt"), str(max_len)]
                           + [c["text"] for c in cases], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        lines = r.stdout.split("\n")
        assert lines[0].startswith("devices ") and lines[0].endswith(" vocab 30522 pad 0")
        got = [[int(v) for v in ln.split()] for ln in lines[1:1 + len(cases)]]
        assert got == [c[key] for c in cases]


def test_tokenizer_entry_points_reject_bad_arguments():
    """The tokenizer's C entry points answer null or negative arguments with
    FUTON_EINVAL or -1 (as futon_tokenizer.h says), never a crash."""
    L = _lib.lib()
    assert L.futon_tokenizer_vocab_size(None) == -1
    assert L.futon_tokenizer_pad_id(None) == -1
    L.futon_tokenizer_destroy(None)
    h = C.c_void_p()
    with pytest.raises(FutonError, match="null argument"):
        _lib.call("futon_tokenizer_create", None, 5, None, C.byref(h))
    with pytest.raises(FutonError, match="null argument"):
        _lib.call("futon_tokenizer_create", b"[CLS]", 5, None, None)
    n = C.c_int(0)
    with pytest.raises(FutonError, match="null or negative"):
        _lib.call("futon_tokenizer_encode", None, b"x", 1, 8, None, 0, C.byref(n))
    cu = (C.c_int32 * 2)()
    with pytest.raises(FutonError, match="null or negative"):
        _lib.call("futon_tokenizer_encode_batch", None, b"x", None, 1, 8, 1, None, 0, cu)
