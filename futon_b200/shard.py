"""Data-parallel sharding of an EmbedBatch across processes (one per GPU).

Every sequence is an independent forward (native/model.go:328-331) and
results are index-aligned (native/provider.go:164-201), so the batch splits
into contiguous sequence ranges with no collective on the data path. The
split balances estimated cost per sequence, L·(12h + 2L) — the dense GEMM
work grows with L, attention with L² — the same rule the library's
multi-device futon_cuda_encode_batch uses inside one process.
"""
from __future__ import annotations

import os
import tempfile
from typing import Callable, List, Tuple

import numpy as np


def sequence_costs(cu_seqlens: np.ndarray, hidden: int) -> np.ndarray:
    L = np.diff(np.asarray(cu_seqlens, dtype=np.float64))
    return L * (12.0 * hidden + 2.0 * L)


def shard_bounds(cu_seqlens: np.ndarray, world: int, hidden: int = 384) -> List[Tuple[int, int]]:
    """Contiguous [s0, s1) sequence ranges, one per rank, balanced by cost."""
    nseq = len(cu_seqlens) - 1
    pref = np.concatenate([[0.0], np.cumsum(sequence_costs(cu_seqlens, hidden))])
    cuts = [0]
    for k in range(1, world):
        target = pref[-1] * k / world
        c = int(np.searchsorted(pref, target, side="left"))
        cuts.append(min(max(c, cuts[-1]), nseq))
    cuts.append(nseq)
    return [(cuts[k], cuts[k + 1]) for k in range(world)]


def shard_for_rank(ids: np.ndarray, cu_seqlens: np.ndarray, rank: int, world: int,
                   hidden: int = 384) -> Tuple[np.ndarray, np.ndarray, int, int]:
    """This rank's (ids, local cu_seqlens, s0, s1)."""
    s0, s1 = shard_bounds(cu_seqlens, world, hidden)[rank]
    t0, t1 = int(cu_seqlens[s0]), int(cu_seqlens[s1])
    return (np.ascontiguousarray(ids[t0:t1]),
            np.ascontiguousarray(cu_seqlens[s0:s1 + 1] - cu_seqlens[s0]).astype(np.int32), s0, s1)


class SharedRows:
    """An index-aligned [rows, dim] float32 host buffer shared by the ranks
    of a process group on one host (a file in /dev/shm mapped by every
    rank): each rank writes its shard's vectors straight into its rows, so
    the result is collected with no copy between processes and no
    collective beyond a barrier. Opening and closing are collective."""

    def __init__(self, rows: int, dim: int, group=None):
        import torch.distributed as dist
        self.group = group
        self.dist = dist.is_initialized() and dist.get_world_size(group) > 1
        rank = dist.get_rank(group) if self.dist else 0
        name = [None]
        if rank == 0:
            base = "/dev/shm" if os.path.isdir("/dev/shm") else tempfile.gettempdir()
            fd, path = tempfile.mkstemp(prefix="futon_rows_", dir=base)
            os.ftruncate(fd, max(1, rows * dim * 4))
            os.close(fd)
            name = [path]
        if self.dist:
            dist.broadcast_object_list(name, src=0, group=group)
        self.path, self.rank = name[0], rank
        self.array = np.memmap(self.path, dtype=np.float32, mode="r+", shape=(rows, dim)) \
            if rows * dim else np.zeros((rows, dim), np.float32)
        self.barrier()

    def barrier(self) -> None:
        if self.dist:
            import torch.distributed as dist
            dist.barrier(group=self.group)

    def close(self) -> None:
        self.barrier()
        self.array = None
        if self.rank == 0 and self.path:
            os.unlink(self.path)
        self.path = None


def embed_batch_shared(encode_into: Callable[[np.ndarray, np.ndarray, np.ndarray], None],
                       ids: np.ndarray, cu_seqlens: np.ndarray, rows: SharedRows,
                       hidden: int = 384) -> Tuple[int, int]:
    """EmbedBatch over a torch.distributed process group, one GPU per rank:
    each rank encodes its cost-balanced shard with `encode_into(ids, cu,
    out)`, writing the vectors into its rows [s0, s1) of `rows`; after the
    closing barrier every rank sees the whole index-aligned result. Returns
    this rank's (s0, s1)."""
    import torch.distributed as dist
    on = dist.is_initialized() and dist.get_world_size(rows.group) > 1
    rank = dist.get_rank(rows.group) if on else 0
    world = dist.get_world_size(rows.group) if on else 1
    sid, scu, s0, s1 = shard_for_rank(ids, cu_seqlens, rank, world, hidden)
    if s1 > s0:
        encode_into(sid, scu, rows.array[s0:s1])
    rows.barrier()
    return s0, s1


def embed_batch_distributed(encode: Callable[[np.ndarray, np.ndarray], np.ndarray],
                            ids: np.ndarray, cu_seqlens: np.ndarray, dim: int,
                            hidden: int = 384, group=None) -> np.ndarray:
    """EmbedBatch over a torch.distributed process group: each rank encodes
    its shard with `encode(ids, cu) -> [n, dim]` (the rank's own GPU) into a
    shared index-aligned host buffer (SharedRows); every rank returns the
    whole [nseq, dim] result."""
    nseq = len(cu_seqlens) - 1
    rows = SharedRows(nseq, dim, group)

    def encode_into(sid, scu, out):
        out[...] = encode(sid, scu)

    embed_batch_shared(encode_into, ids, cu_seqlens, rows, hidden)
    result = np.array(rows.array, dtype=np.float32, copy=True)
    rows.close()
    return result


def max_over_ranks(value: float, group=None) -> float:
    """Max of a per-rank timing (the slowest rank bounds the job)."""
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return value
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
