"""Host-side work partition for one process per GPU.

The attention paths shard without communication except in one place:

  * KDA decode (config 1) and MLA decode (config 4): every rank owns whole sequences
    (weak scaling, no collective on the data path).
  * KDA varlen prefill (config 3): every rank owns a contiguous block of heads for all
    packed sequences; the per-rank outputs [T, H_local, dv] are all-gathered over NVLink
    and interleaved to [T, H, dv] with rank r's heads at r * H_local (the layout the
    reference's o_proj reads, src/core/k3_ops.c:941-949). On the GPU that exchange is
    k3cuda_allgather_heads (NCCL all-gather + an interleave kernel); `gathered_to_heads`
    is the same index map on the host, and `allgather_heads_host` runs it over any
    torch.distributed process group (gloo in the CPU tests).
"""
from __future__ import annotations

import numpy as np


def head_shard(h_total: int, world: int, rank: int) -> slice:
    """Contiguous heads of `rank`; the head count must split evenly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if h_total % world:
        raise ValueError(f"{h_total} heads do not split evenly over {world} ranks")
    per = h_total // world
    return slice(rank * per, (rank + 1) * per)


def sequence_shard(n_seq: int, world: int, rank: int) -> slice:
    """Contiguous sequences of `rank` when a fixed batch is split (remainder to the first
    ranks)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(n_seq, world)
    lo = rank * base + min(rank, extra)
    return slice(lo, lo + base + (1 if rank < extra else 0))


def gathered_to_heads(gathered: np.ndarray) -> np.ndarray:
    """[R, T, H_local, dv] (rank-major, as an all-gather lays it out) -> [T, R*H_local, dv]."""
    R, T, hl, dv = gathered.shape
    return np.ascontiguousarray(gathered.transpose(1, 0, 2, 3).reshape(T, R * hl, dv))


def allgather_heads_host(dist, local: np.ndarray) -> np.ndarray:
    """All-gather this rank's [T, H_local, dv] over `dist` (torch.distributed) and return the
    full [T, H, dv] head layout."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(local))
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t)
    return gathered_to_heads(np.stack([p.numpy() for p in parts]))
