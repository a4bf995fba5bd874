"""Speculative decoding with prompt-lookup (n-gram) drafts, verified greedily by the engine.

vLLM's scheduler feeds each decoding request its newest token followed by the drafts proposed
after the previous step; the engine's call keeps every row of such a request, so it returns the
greedy token after the newest token and after each draft. A draft is accepted while it equals the
token the target chose at its position; the step's output is the accepted drafts' targets plus
one more (the bonus token when every draft is accepted), and vLLM rolls its computed positions
back by the rejected drafts. Keys and values the rejected drafts wrote lie past the accepted
positions, so no later row reads them before a new token overwrites them. The result is exactly
the greedy continuation, whatever the drafts.

Drafts come from vLLM's own `NgramProposer` (prompt lookup over each request's tokens), as in the
reference (integrations/furiosa-opt-vllm/furiosa_opt_vllm/selection.py:40-70 chooses vLLM's
proposers; drafting.py loads a draft model, which is not served here).
"""

from __future__ import annotations

import numpy as np

METHODS = ("ngram",)


def accept(drafts: list[int], targets: list[int]) -> list[int]:
    """The tokens a step produces: `targets[i]` is the greedy token after the row that fed the
    newest token (i = 0) or draft i - 1 (i >= 1), so len(targets) == len(drafts) + 1."""
    if len(targets) != len(drafts) + 1:
        raise ValueError(f"{len(targets)} target tokens for {len(drafts)} drafts")
    out = [int(targets[0])]
    for i, d in enumerate(drafts):
        if int(d) != int(targets[i]):
            break
        out.append(int(targets[i + 1]))
    return out


class Proposer:
    """Proposes each request's next drafts from its tokens (vLLM's n-gram prompt lookup)."""

    def __init__(self, vllm_config):
        from vllm.v1.spec_decode.ngram_proposer import NgramProposer

        self.ngram = NgramProposer(vllm_config)
        self.k = int(vllm_config.speculative_config.num_speculative_tokens)

    def propose(self, sampled: list[list[int]], histories: list[list[int]]) -> list[list[int]]:
        """Drafts per request; a request that produced nothing this step (mid-prompt) gets none."""
        if not histories:
            return []
        width = max(len(h) for h in histories)
        ids = np.zeros((len(histories), max(width, 1)), dtype=np.int32)
        lengths = np.zeros(len(histories), dtype=np.int32)
        for i, h in enumerate(histories):
            ids[i, : len(h)] = h
            lengths[i] = len(h)
        drafts = self.ngram.propose(sampled, lengths, ids)
        return [[int(t) for t in d][: self.k] if s else [] for d, s in zip(drafts, sampled)]
