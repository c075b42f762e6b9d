"""GPU unit parity for the kernel seam (Kernel.MatMulT, MatMulTQ8,
quantizeRowQ8) through the C ABI, mirroring native/kernel_test.go and
native/quant_test.go."""
from __future__ import annotations

import numpy as np
import pytest

from futon_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def naive_matmul_t(a, b, bias):
    out = a.astype(np.float64) @ b.astype(np.float64).T
    if bias is not None:
        out += bias.astype(np.float64)
    return out


# bf16 operands (8-bit mantissa): |err| ≤ 2·2^-9·Σ|a||b| per element, and
# f32 accumulation noise below that; the test bounds by 1e-2 relative to the
# magnitude sum.
@pytest.mark.parametrize("m,n,k", [(1, 8, 8), (3, 4, 16), (7, 16, 32), (13, 29, 64),
                                   (128, 128, 128), (130, 200, 384), (257, 1152, 384),
                                   (300, 384, 1536), (64, 6144, 768)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_matmul_t(gpu, m, n, k, with_bias):
    import torch
    rng = np.random.default_rng(m * 1000 + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32) if with_bias else None
    da, db = _dev(a), _dev(b)
    dbias = _dev(bias) if with_bias else None
    dout = torch.empty((m, n), dtype=torch.float32, device="cuda")
    _lib.call("futon_cuda_matmul_t", 0, dout.data_ptr(), da.data_ptr(), db.data_ptr(), m, n, k,
              dbias.data_ptr() if with_bias else None, None)
    got = dout.cpu().numpy().astype(np.float64)
    want = naive_matmul_t(a, b, bias)
    mag = np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64).T
    assert np.all(np.abs(got - want) <= 1e-2 * mag + 1e-5), np.abs(got - want).max()


@pytest.mark.parametrize("m,n,k", [(1, 1, 16), (2, 3, 32), (5, 9, 64), (13, 29, 128),
                                   (200, 384, 384), (129, 256, 1536), (300, 2304, 768)])
def test_matmul_t_q8_bit_exact(gpu, m, n, k):
    """Q8 GEMM equals the reference scheme bit for bit: same activation
    codes, exact s32 dots, float32(sum)·(sA·sB) + bias (quant.go:99-137)."""
    import torch
    rng = np.random.default_rng(17 + m + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    qb, sb = O.quantize_rows_q8(w)
    want = O.matmul_t_q8(a, qb, sb, bias)
    dout = torch.empty((m, n), dtype=torch.float32, device="cuda")
    # Keep every operand alive across the call (a freed temporary's memory
    # is reused by the caching allocator).
    da, dqb, dsb, dbias = _dev(a), _dev(qb), _dev(sb), _dev(bias)
    _lib.call("futon_cuda_matmul_t_q8", 0, dout.data_ptr(), da.data_ptr(), dqb.data_ptr(),
              dsb.data_ptr(), m, n, k, dbias.data_ptr(), None)
    got = dout.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.abs(got - want).max()


@pytest.mark.parametrize("rows,k", [(1, 4), (3, 257 * 4), (100, 384), (64, 3072)])
def test_quantize_rows_bit_exact(gpu, rows, k):
    import torch
    rng = np.random.default_rng(rows + k)
    x = rng.standard_normal((rows, k)).astype(np.float32)
    x[0, :] = 0.0  # all-zero row: scale 0, zero codes
    if rows > 2:
        x[1, :4] = [0.5, -0.5, 1.5, -2.5]  # halfway cases
    qw, sw = O.quantize_rows_q8(x)
    dq = torch.empty((rows, k), dtype=torch.int8, device="cuda")
    ds = torch.empty(rows, dtype=torch.float32, device="cuda")
    dx = _dev(x)
    _lib.call("futon_cuda_quantize_rows_q8", 0, dq.data_ptr(), ds.data_ptr(), dx.data_ptr(),
              rows, k, None)
    assert np.array_equal(dq.cpu().numpy(), qw)
    assert np.array_equal(ds.cpu().numpy().view(np.uint32), sw.view(np.uint32))
    assert (dq.cpu().numpy() != -128).all()


def test_seam_rejects_bad_shapes(gpu):
    with pytest.raises(_lib.FutonError):
        _lib.call("futon_cuda_matmul_t", 0, None, None, None, 4, 4, 7, None, None)
    with pytest.raises(_lib.FutonError):
        _lib.call("futon_cuda_matmul_t_q8", 0, None, None, None, None, 4, 4, 8, None, None)
    # Well-formed shapes with null buffers are refused on the host.
    with pytest.raises(_lib.FutonError, match="null buffer"):
        _lib.call("futon_cuda_matmul_t", 0, None, None, None, 4, 4, 8, None, None)
    with pytest.raises(_lib.FutonError, match="null buffer"):
        _lib.call("futon_cuda_matmul_t_q8", 0, None, None, None, None, 4, 4, 16, None, None)
    with pytest.raises(_lib.FutonError, match="null buffer"):
        _lib.call("futon_cuda_quantize_rows_q8", 0, None, None, None, 4, 16, None)


def test_seam_concurrent_callers(gpu):
    """Kernel-seam calls from several host threads on one device (the Kernel
    interface is safe for concurrent use): the calls share the device's
    scratch, which grows while they run (the last shape needs more than any
    earlier test), and every result equals the single-threaded one bit for
    bit."""
    import threading

    import torch
    shapes = [(64, 128, 128), (512, 384, 384), (2048, 1152, 384), (8192, 2304, 768)]
    rng = np.random.default_rng(99)
    cases = []
    for m, n, k in shapes:
        a = _dev(rng.standard_normal((m, k)).astype(np.float32))
        b = _dev(rng.standard_normal((n, k)).astype(np.float32))
        cases.append((a, b, m, n, k))

    def run(i, out):
        a, b, m, n, k = cases[i]
        _lib.call("futon_cuda_matmul_t", 0, out.data_ptr(), a.data_ptr(), b.data_ptr(), m, n, k,
                  None, None)

    nthreads, rounds = 4, 2
    outs = [[torch.empty((c[2], c[3]), dtype=torch.float32, device="cuda") for c in cases]
            for _ in range(nthreads)]
    got = [[[] for _ in cases] for _ in range(nthreads)]
    errors = []

    def worker(t):
        try:
            for r in range(rounds):
                order = list(range(len(cases)))
                if (t + r) % 2:
                    order.reverse()
                for i in order:
                    run(i, outs[t][i])
                    got[t][i].append(outs[t][i].cpu().numpy())
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(f"thread {t}: {e!r}")

    threads = [threading.Thread(target=worker, args=(t,)) for t in range(nthreads)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=120)
    assert not any(th.is_alive() for th in threads), "seam calls did not finish"
    assert not errors, errors[:4]
    for i, (a, b, m, n, k) in enumerate(cases):
        ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
        run(i, ref)
        want = ref.cpu().numpy()
        for t in range(nthreads):
            for r, g in enumerate(got[t][i]):
                assert np.array_equal(g, want), f"thread {t} round {r} shape {(m, n, k)}: mismatch"
