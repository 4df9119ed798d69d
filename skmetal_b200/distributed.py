"""Host-side plumbing of multi-GPU fits (one process per GPU).

The data path is sharded by rows: rank ``r`` of ``W`` holds rows
``[n r / W, n (r + 1) / W)`` of the dataset and the library sums the
per-iteration ``k x d`` fixed-point sums and ``k`` counts over the ranks itself
(``skmetal_kmeans_fit_shard``: inside its loop kernel over NVLink, or with an
NCCL all-reduce per iteration when the GPUs cannot map each other's memory). Python only has to give every rank its shard,
create the library's communicator from one NCCL unique id, and reduce timings
over ranks. These helpers take the ``torch.distributed`` module (any backend)
and the bridge as arguments, so the same code runs under NCCL on GPUs and
under gloo in the CPU tests.
"""

from __future__ import annotations

__all__ = ["shard_range", "init_library_comm", "max_over_ranks"]


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Rows ``[lo, hi)`` of rank ``rank``: contiguous, disjoint, covering ``[0, n)``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return (n * rank) // world, (n * (rank + 1)) // world


def init_library_comm(bridge, dist, rank: int, world: int) -> bytes:
    """Create the library's communicator: rank 0 makes the NCCL unique id, every
    rank receives it over ``dist`` and joins. Returns the id."""
    box = [bridge.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    uid = box[0]
    bridge.comm_init(uid, world, rank)
    return uid


def max_over_ranks(dist, values, device="cpu") -> list[float]:
    """Element-wise maximum of a list of floats over all ranks."""
    import torch

    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]
