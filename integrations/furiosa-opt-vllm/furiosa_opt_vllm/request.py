"""Per-request state the runner keeps between steps: the tokens known so far (prompt, then the
tokens it sampled), the history already in the cache, and the block table."""

from __future__ import annotations

import dataclasses

from .paging import BlockTable


@dataclasses.dataclass
class State:
    tokens: list[int]
    prompt: int
    computed: int
    table: BlockTable
    max_tokens: int | None = None
    lora: object = None  # vLLM's LoRARequest of the sequence, or None
    pool: object = None  # pooling.Pool of a pooling request, or None
    # The newest sampled token while it is still on the device: (engine output, row), or None.
    tail: tuple | None = None
    budget: object = None  # thinking.Budget of a request with a thinking-token budget, or None

    def scheduled(self, n: int) -> list[int]:
        """The `n` tokens this step feeds (after the history)."""
        if self.computed + n > len(self.tokens):
            raise ValueError(f"{n} tokens scheduled after {self.computed} of {len(self.tokens)} known")
        return self.tokens[self.computed : self.computed + n]

    def samples_after(self, n: int) -> bool:
        """Whether a step of `n` rows ends at the newest known token (and so samples the next)."""
        return self.computed + n == len(self.tokens)
