"""Speculative decoding with prompt-lookup (n-gram) drafts, verified greedily by the engine.

vLLM's scheduler feeds each decoding request its newest token followed by the drafts proposed
after the previous step; the engine's call keeps every row of such a request, so it returns the
greedy token after the newest token and after each draft. A draft is accepted while it equals the
token the target chose at its position; the step's output is the accepted drafts' targets plus
one more (the bonus token when every draft is accepted), and vLLM rolls its computed positions
back by the rejected drafts. Keys and values the rejected drafts wrote lie past the accepted
positions, so no later row reads them before a new token overwrites them. The result is exactly
the greedy continuation, whatever the drafts.

Drafts come from vLLM's own `NgramProposer` (prompt lookup over each request's tokens), or from a
draft model: a smaller decoder of the same vocabulary loaded beside the target on the worker's
GPU, whose own KV cache is indexed by the target's block tables (the reference chooses vLLM's
proposers in integrations/furiosa-opt-vllm/furiosa_opt_vllm/selection.py:40-70 and loads its
draft model in drafting.py).
"""

from __future__ import annotations

import numpy as np

METHODS = ("ngram", "draft_model")


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

    def attach(self, runner, num_blocks: int) -> None:
        """Prompt lookup keeps no state beside the target."""

    def __init__(self, vllm_config):
        from vllm.v1.spec_decode.ngram_proposer import NgramProposer

        self.ngram = NgramProposer(vllm_config)
        self.k = int(vllm_config.speculative_config.num_speculative_tokens)

    def propose(self, ids: list[str], sampled: list[list[int]], runner) -> list[list[int]]:
        """Drafts per request; a request that produced nothing this step (mid-prompt) gets none."""
        histories = [runner.states[r].tokens for r in ids]
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


class DraftModel:
    """Drafts from a draft model: a decoder of the same vocabulary (its checkpoint is the
    speculative config's `model`) run autoregressively for `num_speculative_tokens` greedy tokens
    after each step of the target.

    The draft's KV cache has the target's block count and is indexed by the target's block tables,
    so a request's positions live in the same blocks in both caches. For each request the draft
    remembers the tokens it has fed; a step feeds the known tokens from the first one that differs
    (the prompt at first, then the accepted tokens), which keeps its cache exactly the request's
    history, then one row a request for each further draft."""

    def __init__(self, vllm_config, load):
        sc = vllm_config.speculative_config
        self.k = int(sc.num_speculative_tokens)
        self.model = load(sc.model)  # path -> engine decoder on the worker's device
        self.cache = None
        self.fed: dict[str, list[int]] = {}

    def attach(self, runner, num_blocks: int) -> None:
        self.cache = runner.dec.Cache(self.model.cache, num_blocks)

    def page_bytes(self) -> int:
        return int(self.model.cache.pools[0].bytes)

    def propose(self, ids: list[str], sampled: list[list[int]], runner) -> list[list[int]]:
        from . import batch

        dec, engine = runner.dec, runner.engine
        live = set(runner.states)
        for rid in [r for r in self.fed if r not in live]:
            del self.fed[rid]
        todo = [i for i, s in enumerate(sampled) if s]
        drafts: list[list[int]] = [[] for _ in ids]
        if not todo or self.k <= 0:
            return drafts
        # First call: every request's tokens the draft has not fed (or fed differently).
        step, hosts, starts = [], [], []
        for i in todo:
            st = runner.states[ids[i]]
            fed = self.fed.get(ids[i], [])
            same = 0
            while same < min(len(fed), len(st.tokens)) and fed[same] == st.tokens[same]:
                same += 1
            same = min(same, len(st.tokens) - 1)  # the newest token is always fed: it predicts the draft
            hosts.append(st.tokens[same:])
            starts.append(same)
            step.append(batch.Scheduled(same, len(st.tokens) - same, len(st.tokens) - same, batch.KEEP_LAST))
        last: list[int] = [0] * len(todo)
        for call in batch.plan(step, int(self.model.rows)):
            flat = np.concatenate([np.asarray(hosts[r.seq][r.offset : r.offset + r.rows], dtype=np.int32) for r in call])
            toks = engine.HostTensor.from_dlpack(flat).to_hbm(runner.device)
            reqs, at = [], 0
            for r in call:
                blocks = runner.states[ids[todo[r.seq]]].table.blocks
                keep = dec.Keep.LAST if r.keep == batch.KEEP_LAST else dec.Keep.NONE
                reqs.append(dec.Request([blocks], r.cached, toks[at : at + r.rows], keep))
                at += r.rows
            out = self.model.forward(reqs, self.cache).to_host().numpy().tolist()
            k = 0
            for r in call:
                if r.keep == batch.KEEP_LAST:
                    last[r.seq] = int(out[k])
                    k += 1
        for j, i in enumerate(todo):
            st = runner.states[ids[i]]
            self.fed[ids[i]] = list(st.tokens)
            drafts[i].append(last[j])
        # Further drafts: one row a request, each feeding the previous draft.
        for _ in range(self.k - 1):
            flat = np.asarray([drafts[i][-1] for i in todo], dtype=np.int32)
            toks = engine.HostTensor.from_dlpack(flat).to_hbm(runner.device)
            reqs = []
            for j, i in enumerate(todo):
                fed = self.fed[ids[i]]
                reqs.append(dec.Request([runner.states[ids[i]].table.blocks], len(fed), toks[j : j + 1], dec.Keep.LAST))
                fed.append(drafts[i][-1])
            out = self.model.forward(reqs, self.cache).to_host().numpy().tolist()
            for j, i in enumerate(todo):
                drafts[i].append(int(out[j]))
        return drafts
