"""A scheduled step as the engine sees it: which rows each request contributes, where its history
starts, and which rows come back (the reference's batch planning,
integrations/furiosa-opt-vllm/furiosa_opt_vllm/batch.py).

Pure host logic, independent of vLLM's classes, so the contract is tested without a framework.
"""

from __future__ import annotations

import dataclasses
from typing import Generic, TypeVar

K = TypeVar("K")


class Framing(ValueError):
    """The framework's token counts do not frame its tokens."""

    def __init__(self, tokens: int, scheduled: int):
        super().__init__(f"{tokens} tokens for {scheduled} scheduled")
        self.tokens = tokens
        self.scheduled = scheduled

    def __reduce__(self):
        return (Framing, (self.tokens, self.scheduled))


@dataclasses.dataclass(frozen=True)
class Row:
    """One scheduled row: its request, the position it writes, whether it is kept."""

    key: object
    position: int
    kept: bool


@dataclasses.dataclass(frozen=True)
class Request(Generic[K]):
    """A request's rows in one call: its history length, its row indices, whether it is kept."""

    key: K
    cached: int
    rows: tuple[int, ...]
    kept: bool


@dataclasses.dataclass(frozen=True)
class Call(Generic[K]):
    requests: tuple[Request[K], ...]
    kept: tuple[int, ...]

    @classmethod
    def plan(cls, rows: tuple[Row, ...], every: bool) -> "Call[K]":
        """Groups consecutive rows of one request (a chunk) in order; keeps the last row of each
        kept request, or every row (pooling) with ``every``."""
        reqs: list[Request] = []
        kept: list[int] = []
        for i, row in enumerate(rows):
            if reqs and reqs[-1].key == row.key and reqs[-1].rows[-1] == i - 1:
                last = reqs[-1]
                reqs[-1] = Request(last.key, last.cached, last.rows + (i,), last.kept or row.kept)
            else:
                reqs.append(Request(row.key, row.position, (i,), row.kept))
            if every or row.kept:
                kept.append(i)
        return cls(tuple(reqs), tuple(kept))


@dataclasses.dataclass(frozen=True)
class Batch:
    """Tokens of each scheduled request (copied, so the framework may reuse its buffers) and the
    history each starts after."""

    tokens: tuple[tuple[int, ...], ...]
    cached: tuple[int, ...]

    @classmethod
    def parse(cls, tokens, lengths, totals) -> "Batch":
        """``tokens`` concatenated per request, ``lengths`` scheduled per request, ``totals`` the
        positions each request reaches after the step."""
        if len(lengths) != len(totals):
            raise Framing(len(tokens), sum(lengths))
        if any(n <= 0 for n in lengths) or any(t < n for n, t in zip(lengths, totals)):
            raise Framing(len(tokens), sum(max(n, 0) for n in lengths))
        if sum(lengths) != len(tokens):
            raise Framing(len(tokens), sum(lengths))
        out, at = [], 0
        for n in lengths:
            out.append(tuple(int(t) for t in tokens[at : at + n]))
            at += n
        return cls(tuple(out), tuple(t - n for n, t in zip(lengths, totals)))
