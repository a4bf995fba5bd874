"""A minimal serving loop over the public engine API: the framework side of a call (block
assignment, prompt chunking, greedy decode), as the vLLM and SGLang plugins drive it.

The engine owns cache storage and the calls; this module owns which blocks each sequence holds
and what each call contains (the reference's split: the framework schedules, the engine runs).
"""

from __future__ import annotations

import dataclasses

import furiosa_opt_engine as engine
from furiosa_opt_engine import decoder as dec


class BlockAllocator:
    """Free block IDs of one cache (a stack: recently freed blocks are reused first)."""

    def __init__(self, blocks: int):
        self.free = list(range(blocks - 1, -1, -1))

    def take(self, n: int) -> list[int]:
        if n > len(self.free):
            raise RuntimeError(f"cache has {len(self.free)} free blocks, {n} wanted")
        out = self.free[-n:][::-1] if n else []
        del self.free[len(self.free) - n :]
        return out

    def give(self, ids: list[int]) -> None:
        self.free.extend(reversed(ids))


@dataclasses.dataclass
class Sequence:
    prompt: engine.HbmTensor  # I32 prompt IDs on the device
    length: int
    blocks: list[int]
    cached: int = 0
    last: engine.HbmTensor | None = None  # the newest token, on the device
    produced: int = 0


def blocks_for(positions: int, block: int = 16) -> int:
    return (positions + block - 1) // block


def prefill_calls(seqs: list[Sequence], rows: int) -> list[list[int]]:
    """Indices of sequences per prefill call: whole prompts packed up to `rows` rows a call."""
    calls, cur, used = [], [], 0
    for i, s in enumerate(seqs):
        if cur and used + s.length > rows:
            calls.append(cur)
            cur, used = [], 0
        cur.append(i)
        used += s.length
    if cur:
        calls.append(cur)
    return calls


def prefill(model, cache, seqs: list[Sequence], call: list[int]) -> engine.HbmTensor:
    """One prefill call of whole prompts; each sequence's first token becomes its `last`."""
    reqs = [dec.Request([seqs[i].blocks], 0, seqs[i].prompt, dec.Keep.LAST) for i in call]
    out = model.forward(reqs, cache)
    for k, i in enumerate(call):
        seqs[i].cached = seqs[i].length
        seqs[i].last = out[k : k + 1]
        seqs[i].produced = 1
    return out


def decode(model, cache, seqs: list[Sequence]) -> engine.HbmTensor:
    """One decode step of every sequence: its newest token appended, the next one returned."""
    reqs = [dec.Request([s.blocks], s.cached, s.last, dec.Keep.LAST) for s in seqs]
    out = model.forward(reqs, cache)
    for k, s in enumerate(seqs):
        s.cached += 1
        s.last = out[k : k + 1]
        s.produced += 1
    return out
