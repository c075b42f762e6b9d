"""The Q8 GEMM entry point that allocates nothing.

Some callers must not allocate device memory while they run — a serving loop
whose GPU memory another allocator already holds, or a latency-critical path
where cudaMalloc/cudaFree (which synchronises the device) is not allowed.
futon_cuda_matmul_t_q8_noalloc serves them from a fixed 4 MiB device array
instead of library scratch. It must give exactly the results of
futon_cuda_matmul_t_q8 (the Q8 scheme is integer-exact), call after call,
and refuse shapes that do not fit the array.
"""
from __future__ import annotations

import numpy as np
import pytest

from futon_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _run(fn, m, n, k, seed):
    import torch
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    qb, sb = O.quantize_rows_q8(w)
    # All operands stay referenced until the call returns.
    da = torch.from_numpy(a).cuda()
    dqb = torch.from_numpy(qb).cuda()
    dsb = torch.from_numpy(sb).cuda()
    dbias = torch.from_numpy(bias).cuda()
    dout = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    _lib.call(fn, 0, dout.data_ptr(), da.data_ptr(), dqb.data_ptr(), dsb.data_ptr(), m, n, k,
              dbias.data_ptr(), None)
    return dout.cpu().numpy()


@pytest.mark.parametrize("first,second", [((200, 384, 384), (96, 2304, 768)),
                                          ((1024, 3072, 3072), (7, 16, 32))])
def test_noalloc_matches_allocating_entry_point(gpu, first, second):
    """Two calls in a row, each equal bit for bit to futon_cuda_matmul_t_q8
    on the same inputs (the second call overwrites the shared array)."""
    for i, (m, n, k) in enumerate((first, second)):
        got = _run("futon_cuda_matmul_t_q8_noalloc", m, n, k, seed=100 + i)
        want = _run("futon_cuda_matmul_t_q8", m, n, k, seed=100 + i)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (m, n, k)


def test_noalloc_rejects_oversized(gpu):
    with pytest.raises(_lib.FutonError, match="no-alloc scratch"):
        _lib.call("futon_cuda_matmul_t_q8_noalloc", 0, None, None, None, None, 2048, 64, 3072,
                  None, None)
