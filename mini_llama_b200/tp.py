"""Tensor-parallel plumbing for the batched decode driver: one process per GPU,
rendezvous and the NCCL id exchange over torch.distributed (any backend; the
collectives of the decode step itself run inside the library over NCCL)."""
from __future__ import annotations

from typing import Callable


def share_nccl_id(dist, make_id: Callable[[], bytes]) -> bytes:
    """Rank 0 makes the id; every rank of the default group receives it."""
    obj = [make_id() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    nid = obj[0]
    if not isinstance(nid, (bytes, bytearray)) or len(nid) != 128:
        raise RuntimeError("NCCL id exchange returned a malformed id")
    return bytes(nid)


def max_over_ranks(dist, values: list[float]) -> list[float]:
    """Element-wise maximum of per-rank host timings (CPU tensor all-reduce)."""
    import torch
    t = torch.tensor(values, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]
