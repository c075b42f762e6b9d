"""Data-parallel sharding across processes, on CPU with gloo (world size 2):
the shards tile the batch, balance cost, and the gathered result equals the
single-process result bit for bit (the CPU oracle stands in for each rank's
GPU, exactly like the GPU ranks would run their own replicas)."""
from __future__ import annotations

import os
import socket

import numpy as np
import torch.multiprocessing as mp

from conftest import GOLDEN
from futon_b200 import synth
from futon_b200.shard import sequence_costs, shard_bounds, shard_for_rank


def test_bounds_tile_and_balance():
    ids, cu = synth.make_inputs("c4", nseq=4096)
    for world in (1, 2, 3, 4, 8):
        b = shard_bounds(cu, world)
        assert b[0][0] == 0 and b[-1][1] == 4096
        assert all(b[k][1] == b[k + 1][0] for k in range(world - 1))
        costs = sequence_costs(cu, 384)
        per = np.array([costs[s0:s1].sum() for s0, s1 in b])
        assert per.max() <= per.sum() / world + costs.max() + 1e-6


def test_bounds_properties_random():
    """Any lengths and world size (more ranks than sequences included): the
    ranges are contiguous, cover every sequence once, and no rank carries
    more than its even share plus one sequence's cost."""
    from hypothesis import given, settings
    from hypothesis import strategies as st

    @settings(max_examples=200, deadline=None)
    @given(st.lists(st.integers(1, 2048), min_size=0, max_size=64), st.integers(1, 12))
    def check(lens, world):
        cu = np.zeros(len(lens) + 1, np.int32)
        np.cumsum(lens, out=cu[1:])
        b = shard_bounds(cu, world)
        assert len(b) == world and b[0][0] == 0 and b[-1][1] == len(lens)
        assert all(b[k][1] == b[k + 1][0] for k in range(world - 1))
        assert all(s0 <= s1 for s0, s1 in b)
        if lens:
            costs = sequence_costs(cu, 384)
            per = np.array([costs[s0:s1].sum() for s0, s1 in b])
            assert per.max() <= per.sum() / world + costs.max() * (1 + 1e-9) + 1e-6

    check()


def test_shard_for_rank_local_offsets():
    ids, cu = synth.make_inputs("c4", nseq=50)
    got = []
    for r in range(3):
        sid, scu, s0, s1 = shard_for_rank(ids, cu, r, 3)
        assert scu[0] == 0 and scu[-1] == len(sid)
        got.append(sid)
    assert np.array_equal(np.concatenate(got), ids)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_path):
    import torch.distributed as dist
    from futon_b200.pack import load_pack
    from futon_b200.shard import embed_batch_distributed, max_over_ranks
    from oracle.oracle import OracleModel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    pk = load_pack(GOLDEN / "toy-rope-swiglu", keep_f16=False)
    m = OracleModel(pk.cfg, pk.tensors)
    rng = np.random.default_rng(0)
    lens = rng.integers(2, 40, size=11)
    seqs = [rng.integers(0, pk.cfg.vocab_size, L) for L in lens]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    ids = np.concatenate(seqs).astype(np.int32)
    out = embed_batch_distributed(lambda i, c: m.encode_batch(i, c, threads=1), ids, cu,
                                  pk.cfg.hidden_size, hidden=pk.cfg.hidden_size)
    t = max_over_ranks(float(rank + 1))
    if rank == 0:
        np.save(result_path, out)
        np.save(result_path + ".t.npy", np.array([t]))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks_match_single(tmp_path):
    from futon_b200.pack import load_pack
    from oracle.oracle import OracleModel
    path = str(tmp_path / "out.npy")
    mp.start_processes(_worker, args=(2, _free_port(), path), nprocs=2, join=True,
                       start_method="spawn")
    got = np.load(path)
    assert float(np.load(path + ".t.npy")[0]) == 2.0
    pk = load_pack(GOLDEN / "toy-rope-swiglu", keep_f16=False)
    m = OracleModel(pk.cfg, pk.tensors)
    rng = np.random.default_rng(0)
    lens = rng.integers(2, 40, size=11)
    seqs = [rng.integers(0, pk.cfg.vocab_size, L) for L in lens]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    want = m.encode_batch(np.concatenate(seqs).astype(np.int32), cu, threads=1)
    assert np.array_equal(got, want)
