"""Tensor-parallel plumbing of a loaded decoder.

Each rank (one process per GPU) allocates a symmetric heap for the fused collectives, exports it
as a CUDA IPC handle, and opens every peer's handle after an all-gather over the process group.
From then on each row-parallel projection writes its FP32 partial locally, the partial is stored
over NVLink into the receive slots of the ranks that reduce it (by a scatter kernel, or in small
calls by the reducer itself), and the reducer adds the ranks' partials in rank order with the
residual and applies the next RMSNorm; the vocabulary-parallel head ends in an exchange of
(value, token) candidates. `emulate.py` runs the same schedule on the host as its oracle.
"""

from __future__ import annotations

# The process group a placement's ranks form (None: the default group). A framework that runs
# several replicas in one group (data parallelism) names each replica's tensor-parallel group.
_group = None


def set_group(group) -> None:
    global _group
    _group = group


def rank_for_chips(chips: int) -> int:
    """This process's rank among the `chips` processes of a placement (one process per GPU, process
    `rank` serving `chips[rank]`), from the process group when it is up, else from RANK and
    WORLD_SIZE; raises when the group's size is not the placement's. `engine.Device` calls it."""
    import os

    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        world, rank = dist.get_world_size(_group), dist.get_rank(_group)
    else:
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
    if world != chips:
        raise RuntimeError(f"a placement of {chips} chips runs as {chips} processes, one per GPU; this group has {world}")
    return rank


def exchange_handles(handle: bytes) -> list:
    """Every rank's heap handle, in rank order. A rank that has died or never joins ends the
    exchange with the process group's error (its timeout bounds the wait), before any kernel of
    this rank waits on that peer."""
    import torch.distributed as dist

    handles: list = [None] * dist.get_world_size(_group)
    dist.all_gather_object(handles, handle, group=_group)
    if any(h is None for h in handles):
        raise RuntimeError("a rank gave no tensor-parallel heap handle")
    return handles


def attach(model, device) -> None:
    """Connects `model` (this rank's shard) to its peers; every rank calls it, in the same order."""
    import torch.distributed as dist

    from furiosa_opt_engine import _native

    world, rank = dist.get_world_size(_group), dist.get_rank(_group)
    handle = _native._tp_attach(model, world, rank)
    handles = exchange_handles(handle)
    _native._tp_connect(model, handles)
    dist.barrier(group=_group)
    # A device-side barrier through the heaps proves every peer mapping works before any call.
    _native._tp_barrier(model)
    dist.barrier(group=_group)


def detach(model) -> None:
    """Releases the heap once every rank has stopped using it."""
    import torch.distributed as dist

    from furiosa_opt_engine import _native

    model.device.synchronize()
    dist.barrier(group=_group)
    _native._tp_detach(model)
    dist.barrier(group=_group)
