"""Process-group plumbing: which chip of a placement this process serves.

A placement of N chips runs as N processes, one per GPU (launched by ``torchrun`` or any launcher
that sets RANK/WORLD_SIZE), joined in a ``torch.distributed`` group over NCCL. Process ``rank``
serves ``chips[rank]``.
"""

from __future__ import annotations

import os


def rank_for_chips(chips: int) -> int:
    """This process's rank among ``chips`` processes; raises when the group does not match."""
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        world, rank = dist.get_world_size(), dist.get_rank()
    else:
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
    if world != chips:
        raise RuntimeError(
            f"a placement of {chips} chips runs as {chips} processes, one per GPU; "
            f"this group has {world}"
        )
    return rank
