"""SGLang's KV pool as engine blocks.

SGLang addresses its KV pool by token slot: ``req_to_token[req, position]`` is the slot of a
request's token. With ``page_size`` 16 a page holds 16 consecutive slots, so slot // 16 is the
engine's block ID and the page of position p of a request is req_to_token[req, 16 * (p // 16)]
// 16 (the reference's paging: integrations/furiosa-opt-sglang/furiosa_opt_sglang/paging.py).
"""

from __future__ import annotations

PAGE = 16


class Misaligned(ValueError):
    """A request's slots do not fill whole pages in order."""


def blocks(slots, positions: int) -> list[int]:
    """The blocks of a request's first `positions` positions from its slot row (any sequence of
    ints indexable by position)."""
    out = []
    for start in range(0, positions, PAGE):
        s = int(slots[start])
        if s % PAGE != 0:
            raise Misaligned(f"position {start} sits in slot {s}, not at a page start")
        out.append(s // PAGE)
    return out


def check_page_size(page_size: int) -> None:
    if page_size != PAGE:
        raise ValueError(f"page_size {page_size}: the engine's cache pages hold {PAGE} tokens")


def assign(req_pool_indices, req_to_token, start_offset, end_offset, out_cache_loc, batch_size: int) -> None:
    """Writes each request's new token slots into its row of the host request table (SGLang's
    `assign_req_to_token_pool_func` contract: request i's slots for positions start..end follow
    the earlier requests' in `out_cache_loc`)."""
    at = 0
    for i in range(int(batch_size)):
        start, end = int(start_offset[i]), int(end_offset[i])
        req_to_token[int(req_pool_indices[i]), start:end] = out_cache_loc[at : at + end - start]
        at += end - start
