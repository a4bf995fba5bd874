"""Block tables: vLLM's KV cache manager hands out block IDs per request; the engine reads the
same IDs as its pool's block indices (one group, 16-token blocks)."""

from __future__ import annotations

BLOCK = 16


class BlockTable:
    """One request's blocks, grown as vLLM appends (and replaced when a preempted request
    resumes)."""

    def __init__(self, blocks=()):
        self.blocks: list[int] = list(blocks)

    def append(self, blocks) -> None:
        self.blocks.extend(int(b) for b in blocks)

    def replace(self, blocks) -> None:
        self.blocks = [int(b) for b in blocks]

    def covers(self, positions: int) -> bool:
        return len(self.blocks) * BLOCK >= positions


def first_group(block_ids) -> list[int]:
    """vLLM's block IDs per KV cache group: the engine's decoders use one group."""
    if block_ids is None:
        return []
    if len(block_ids) != 1:
        raise ValueError(f"{len(block_ids)} KV cache groups; the engine's decoders use one")
    return list(block_ids[0])
