"""A forward batch as the engine sees it. SGLang describes a batch by its requests' pool rows,
their lengths after the batch, the prefix already cached and the new tokens (extend), or one new
token each (decode); this module turns those fields into engine requests, independent of SGLang's
classes (the reference's batch planning:
integrations/furiosa-opt-sglang/furiosa_opt_sglang/batch.py)."""

from __future__ import annotations

import dataclasses

from . import paging


@dataclasses.dataclass(frozen=True)
class Part:
    """One request of a batch: its pool row, the cached history, its new tokens' span in the
    batch's flat token list, whether its last row is returned."""

    row: int
    cached: int
    start: int
    count: int
    keep: bool


def parts(req_rows, seq_lens, prefix_lens, new_lens, keep_last=True) -> list[Part]:
    """Requests of a batch: ``seq_lens`` after the batch, ``prefix_lens`` cached before it,
    ``new_lens`` tokens each contributes (extend), in batch order."""
    out, at = [], 0
    for row, total, cached, n in zip(req_rows, seq_lens, prefix_lens, new_lens):
        total, cached, n = int(total), int(cached), int(n)
        if n <= 0 or cached + n != total:
            raise ValueError(f"request row {row}: {cached} cached + {n} new != {total}")
        out.append(Part(int(row), cached, at, n, keep_last))
        at += n
    return out


def decode_parts(req_rows, seq_lens) -> list[Part]:
    """A decode batch: one new token per request after its seq_len - 1 cached positions."""
    return [Part(int(r), int(t) - 1, i, 1, True) for i, (r, t) in enumerate(zip(req_rows, seq_lens))]


def request_blocks(req_to_token, part: Part) -> list[int]:
    """The engine blocks a part's positions live in (its whole history and new tokens)."""
    return paging.blocks(req_to_token[part.row], part.cached + part.count)
