"""Data-parallel sharding of an EmbedBatch across processes (one per GPU).

Every sequence is an independent forward (native/model.go:328-331) and
results are index-aligned (native/provider.go:164-201), so the batch splits
into contiguous sequence ranges with no collective on the data path. The
split balances estimated cost per sequence, L·(12h + 2L) — the dense GEMM
work grows with L, attention with L² — the same rule the library's
multi-device futon_cuda_encode_batch uses inside one process.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Tuple

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


def embed_batch_distributed(encode: Callable[[np.ndarray, np.ndarray], np.ndarray],
                            ids: np.ndarray, cu_seqlens: np.ndarray, dim: int,
                            hidden: int = 384, group=None) -> np.ndarray:
    """EmbedBatch over a torch.distributed process group: each rank encodes
    its shard with `encode(ids, cu) -> [n, dim]` (the rank's own GPU), then
    the shards are all-gathered into the index-aligned [nseq, dim] result.
    The gather is result collection only (vectors back to the caller), not
    part of the forward."""
    import torch
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    sid, scu, s0, s1 = shard_for_rank(ids, cu_seqlens, rank, world, hidden)
    local = encode(sid, scu) if s1 > s0 else np.zeros((0, dim), np.float32)
    parts: List[Optional[np.ndarray]] = [None] * world
    dist.all_gather_object(parts, np.ascontiguousarray(local, dtype=np.float32), group=group)
    out = np.concatenate([p for p in parts if p is not None and len(p)], axis=0) \
        if any(p is not None and len(p) for p in parts) else np.zeros((0, dim), np.float32)
    assert out.shape[0] == len(cu_seqlens) - 1
    return out


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
