"""Several GPUs in one process: futon_cuda_encode_batch shards a batch into
contiguous cost-balanced sequence ranges, one host thread, stream and weight
replica per device, and writes every vector to its index (the
EmbedBatch contract, native/provider.go:152-246). No collective is involved,
so each vector must equal, bit for bit, what one device computes for it.
Skipped on boxes with fewer than two GPUs."""
from __future__ import annotations

import numpy as np
import pytest

from futon_b200 import _lib, synth
from futon_b200.provider import Model

pytestmark = pytest.mark.gpu


def _ndev() -> int:
    return int(_lib.lib().futon_cuda_device_count())


@pytest.mark.parametrize("arch", ["bge", "nomic"])
def test_encode_batch_across_devices_matches_one(gpu, arch):
    n = _ndev()
    if n < 2:
        pytest.skip("needs two or more GPUs")
    cfg = synth.arch(arch)
    cfg.num_layers = 3
    w = synth.make_weights(cfg)
    ids, cu = synth.make_inputs("c4" if arch == "bge" else "c2", nseq=300, seed=7,
                                vocab=cfg.vocab_size)
    one = Model(cfg, w, devices=[0])
    many = Model(cfg, w, devices=list(range(n)))
    want = one.encode_packed(ids, cu)
    got = many.encode_batch(ids, cu)
    assert got.shape == want.shape
    assert np.array_equal(got, want)
    one.close()
    many.close()
