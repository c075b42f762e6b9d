"""Failure detection on the device, tested without a GPU fault.

Every pipeline kernel bounds its mbarrier waits (1 s); a wait that runs out
records a code in the device error word, raises the CTA's abort flag and the
kernel returns, so the host reports FUTON_EDEVICE and the CUDA context stays
usable. futon_cuda_selftest_wait_timeout runs that routine against a barrier
phase that nothing completes; the test checks the reported status and that
the library still computes correct results afterwards.
"""
from __future__ import annotations

import numpy as np
import pytest

from futon_b200 import _lib, synth
from futon_b200.provider import Model

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_context_survives(gpu):
    with pytest.raises(_lib.FutonError) as ei:
        _lib.call("futon_cuda_selftest_wait_timeout", 0)
    assert ei.value.code == _lib.FUTON_EDEVICE
    assert "timed out" in str(ei.value)

    # The device is still usable: a forward runs and matches a second run.
    cfg = synth.arch("bge")
    cfg.num_layers = 2
    m = Model(cfg, synth.make_weights(cfg), devices=[0])
    ids, cu = synth.make_inputs("c0", nseq=4, seed=5)
    a = m.encode_packed(ids, cu)
    b = m.encode_packed(ids, cu)
    assert np.array_equal(a, b)
    assert np.allclose(np.linalg.norm(a, axis=1), 1.0, atol=1e-5)
    m.close()
