"""The Q8 GEMM entry point that allocates nothing.

Some callers must not allocate device memory while they run — a serving loop
whose GPU memory another allocator already holds, or a latency-critical path
where cudaMalloc/cudaFree (which synchronises the device) is not allowed.
futon_cuda_matmul_t_q8_noalloc serves them from a fixed 4 MiB device array
instead of library scratch. It must give exactly the results of
futon_cuda_matmul_t_q8 and of the reference's Q8 scheme (integer-exact dots,
float32(sum)·(sA·sB) + bias), call after call, leave the device's free
memory unchanged once its device code is loaded, and refuse shapes that do
not fit the array.
"""
from __future__ import annotations

import numpy as np
import pytest

from futon_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu

# Shapes whose scalar oracle GEMM finishes in about a second.
ORACLE_MAX_MACS = 2e8


def _inputs(m, n, k, seed):
    import torch
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    qb, sb = O.quantize_rows_q8(w)
    host = (a, qb, sb, bias)
    # All operands stay referenced until the caller is done with the call.
    dev = [torch.from_numpy(x).cuda() for x in host]
    dout = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    return host, dev, dout


def _call(fn, m, n, k, dev, dout):
    da, dqb, dsb, dbias = dev
    _lib.call(fn, 0, dout.data_ptr(), da.data_ptr(), dqb.data_ptr(), dsb.data_ptr(), m, n, k,
              dbias.data_ptr(), None)


def _run(fn, m, n, k, seed):
    host, dev, dout = _inputs(m, n, k, seed)
    _call(fn, m, n, k, dev, dout)
    return host, dout.cpu().numpy()


def test_noalloc_leaves_free_memory_unchanged(gpu):
    """After one warm-up call per shape (which loads the library's device
    code, and with it the fixed array, if no earlier call did), further
    calls of those shapes change the device's free memory by nothing."""
    import torch
    shapes = [(200, 384, 384), (1024, 3072, 3072), (7, 16, 32)]
    prepared = [(s, *_inputs(*s, seed=7 + i)[1:]) for i, s in enumerate(shapes)]
    for (m, n, k), dev, dout in prepared:
        _call("futon_cuda_matmul_t_q8_noalloc", m, n, k, dev, dout)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        for (m, n, k), dev, dout in prepared:
            _call("futon_cuda_matmul_t_q8_noalloc", m, n, k, dev, dout)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"free device memory moved by {free0 - free1} bytes"


@pytest.mark.parametrize("first,second", [((200, 384, 384), (96, 2304, 768)),
                                          ((1024, 3072, 3072), (7, 16, 32))])
def test_noalloc_matches_allocating_entry_point(gpu, first, second):
    """Two calls in a row, each equal bit for bit to futon_cuda_matmul_t_q8
    on the same inputs (the second call overwrites the shared array), and to
    the CPU oracle's Q8 GEMM (quant.go:99-137) where that finishes quickly."""
    for i, (m, n, k) in enumerate((first, second)):
        (a, qb, sb, bias), got = _run("futon_cuda_matmul_t_q8_noalloc", m, n, k, seed=100 + i)
        _, want = _run("futon_cuda_matmul_t_q8", m, n, k, seed=100 + i)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (m, n, k)
        if m * n * k <= ORACLE_MAX_MACS:
            ref = O.matmul_t_q8(a, qb, sb, bias)
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (m, n, k)


def test_noalloc_rejects_oversized(gpu):
    with pytest.raises(_lib.FutonError, match="no-alloc scratch"):
        _lib.call("futon_cuda_matmul_t_q8_noalloc", 0, None, None, None, None, 2048, 64, 3072,
                  None, None)
