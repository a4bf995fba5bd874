"""SGLang's speculative decoding through the engine: n-gram (NGRAM) and draft-model (STANDALONE)
drafts, verified greedily by the target.

SGLang's speculative schedule is synchronous: each step's result is processed before the next step
is issued. A prompt (extend) step runs as usual and commits one token a request. A decode step
builds one chain a request: its last token followed by up to `width - 1` drafts (fewer where the
context ends). The target runs every chain in calls of at most `rows` rows and keeps every chain
row (`Keep.ALL`), so it returns its greedy token after each; a draft is accepted while it equals
the target's token at the position before it, and the request commits the accepted drafts plus
the target's token after the last of them. The committed tokens are the greedy continuation
whatever the drafts were. Keys and values that rejected drafts wrote lie past the committed
positions, where the next token's row overwrites them before any row reads them.

SGLang reads a step's committed tokens at a stride of the verification width (`next_token_ids`)
with their counts (`accept_lens`), advances its sequence lengths (`new_seq_lens`), and carries the
same fields in the step's `next_draft_input`. The result fields and the worker's constructor are
SGLang's speculative-worker interface, as the reference plugin serves it
(integrations/furiosa-opt-sglang/furiosa_opt_sglang/speculative/__init__.py, ngram.py,
standalone.py).

Nothing here imports SGLang at module load: `worker_class()` subclasses SGLang's `BaseSpecWorker`
when SGLang is importable.
"""

from __future__ import annotations

import dataclasses

import numpy as np

from . import steps

ALGORITHMS = ("NGRAM", "STANDALONE")


@dataclasses.dataclass(frozen=True)
class Decoding:
    """A decoding request as a proposer reads it: its tokens (the target caches all but the last),
    the most drafts its context leaves room for, and its request-pool row."""

    rid: str
    tokens: tuple[int, ...]
    drafts: int
    slot: int

    @property
    def cached(self) -> int:
        return len(self.tokens) - 1


def accept(chain: tuple[int, ...], targets: list[int]) -> tuple[int, ...]:
    """The tokens a chain commits: `targets[i]` is the target's greedy token after chain row i (the
    last token for i = 0, draft i otherwise)."""
    if len(targets) != len(chain):
        raise ValueError(f"{len(targets)} target tokens for a chain of {len(chain)}")
    kept = 0
    while kept + 1 < len(chain) and chain[kept + 1] == targets[kept]:
        kept += 1
    return tuple(int(t) for t in targets[: kept + 1])


class Ngram:
    """Drafts from each request's own tokens: the longest suffix of `max_n` down to `min_n` tokens
    that occurred earlier, and the tokens that followed its latest earlier occurrence."""

    def __init__(self, k: int, min_n: int = 1, max_n: int = 3):
        if k < 1 or min_n < 1 or max_n < min_n:
            raise ValueError(f"n-gram drafting needs k >= 1 and 1 <= min_n <= max_n (k={k}, {min_n}..{max_n})")
        self.k, self.min_n, self.max_n = k, min_n, max_n

    def propose(self, runner, decodings: list[Decoding], req_to_token) -> list[list[int]]:
        return [self.draft(d.tokens, min(self.k, d.drafts)) for d in decodings]

    def draft(self, tokens, k: int) -> list[int]:
        a = np.asarray(tokens, dtype=np.int64)
        if k <= 0:
            return []
        for n in range(min(self.max_n, len(a) - 1), self.min_n - 1, -1):
            # Windows of n tokens that end before the last token, each followed by at least one.
            windows = np.lib.stride_tricks.sliding_window_view(a[:-1], n)
            hits = np.nonzero((windows == a[-n:]).all(axis=1))[0]
            if len(hits):
                start = int(hits[-1]) + n
                return [int(t) for t in a[start : start + k]]
        return []

    def committed(self, rid: str, tokens: tuple[int, ...]) -> None:
        """Prompt lookup keeps no state."""

    def forget(self, rids) -> None:
        pass

    def reset(self) -> None:
        pass


class DraftModel:
    """Drafts from a draft model: a smaller decoder of the same vocabulary, run greedily for `k`
    tokens a step. Its KV cache has the target's block count and is indexed by the target's page
    tables, so a request's positions live in the same blocks of both caches. For each request the
    draft remembers the tokens whose keys and values its cache holds; a step feeds the request's
    tokens from the first one it does not hold (the whole prompt at first, then the committed
    tokens), then one row a request for each further draft."""

    def __init__(self, model, cache, k: int):
        if k < 1:
            raise ValueError("a draft model proposes at least one token")
        self.model, self.cache, self.k = model, cache, k
        self.held: dict[str, tuple[int, ...]] = {}

    def propose(self, runner, decodings: list[Decoding], req_to_token) -> list[list[int]]:
        ks = [min(self.k, d.drafts) for d in decodings]
        todo = [i for i, k in enumerate(ks) if k > 0]
        drafts: list[list[int]] = [[] for _ in decodings]
        if not todo:
            return drafts
        # First call: each request's tokens from the first one the draft cache does not hold; the
        # last token is always fed, since its row predicts the first draft.
        firsts = []
        for i in todo:
            d = decodings[i]
            held = self.held.get(d.rid, ())
            same = 0
            while same < min(len(held), len(d.tokens)) and held[same] == d.tokens[same]:
                same += 1
            firsts.append(min(same, len(d.tokens) - 1))
        lengths = [len(decodings[i].tokens) - f for i, f in zip(todo, firsts)]
        last = self._run(runner, req_to_token, [decodings[i] for i in todo], firsts, lengths,
                         [decodings[i].tokens[f:] for i, f in zip(todo, firsts)])
        for j, i in enumerate(todo):
            self.held[decodings[i].rid] = decodings[i].tokens
            drafts[i].append(last[j])
        # Further drafts: one row a request, each feeding the previous draft.
        for step in range(1, max(ks)):
            more = [i for i in todo if ks[i] > step]
            if not more:
                break
            got = self._run(runner, req_to_token, [decodings[i] for i in more],
                            [len(decodings[i].tokens) + step - 1 for i in more], [1] * len(more),
                            [(drafts[i][-1],) for i in more])
            for j, i in enumerate(more):
                self.held[decodings[i].rid] = self.held[decodings[i].rid] + (drafts[i][-1],)
                drafts[i].append(got[j])
        return drafts

    def _run(self, runner, req_to_token, decodings, cached, lengths, tokens) -> list[int]:
        """Feeds `tokens[i]` after `cached[i]` positions of each request; returns the draft's greedy
        token after each request's last fed row."""
        out = [0] * len(decodings)
        for call in steps.plan(lengths, cached, int(self.model.rows)):
            flat = np.concatenate([np.asarray(tokens[r.seq][r.first : r.first + r.count], dtype=np.int32)
                                   for r in call])
            dev = runner.engine.HostTensor.from_dlpack(np.ascontiguousarray(flat)).to_hbm(runner.device)
            reqs, at, kept = [], 0, []
            for r in call:
                blocks = runner.blocks(req_to_token, decodings[r.seq].slot, r.cached + r.count)
                keep = runner.dec.Keep.LAST if r.last else runner.dec.Keep.NONE
                reqs.append(runner.dec.Request([blocks], r.cached, dev[at : at + r.count], keep))
                at += r.count
                if r.last:
                    kept.append(r.seq)
            host = np.asarray(self.model.forward(reqs, self.cache).to_host().numpy()).reshape(-1)
            for row, s in enumerate(kept):
                out[s] = int(host[row])
        return out

    def committed(self, rid: str, tokens: tuple[int, ...]) -> None:
        """Keeps what the draft cache holds of the request's committed tokens: its rows of rejected
        drafts no longer match and are fed again."""
        held = self.held.get(rid)
        if held is None:
            return
        same = 0
        while same < min(len(held), len(tokens)) and held[same] == tokens[same]:
            same += 1
        self.held[rid] = tokens[:same]

    def forget(self, rids) -> None:
        for r in rids:
            self.held.pop(r, None)

    def reset(self) -> None:
        self.held.clear()


@dataclasses.dataclass
class Speculation:
    """A target's speculative decoding: the proposer and the verification width (the last token
    and the drafts after it)."""

    proposer: object
    width: int

    def decode(self, runner, batch, req_to_token, context: int):
        """A decode step: chains, one verification, the committed tokens of each request."""
        slots = steps._ints(batch.req_pool_indices)
        seq_lens = steps._ints(batch.seq_lens)
        decodings = []
        for req, slot, cached in zip(batch.reqs, slots, seq_lens):
            tokens = tuple(int(t) for t in (*req.origin_input_ids, *req.output_ids))
            if cached != len(tokens) - 1:
                raise ValueError(f"{req.rid}: SGLang caches {cached} of the request's {len(tokens)} tokens")
            room = max(1, min(self.width, context - cached))
            decodings.append(Decoding(req.rid, tokens, room - 1, slot))
        chains = [(d.tokens[-1], *drafts[: d.drafts])
                  for d, drafts in zip(decodings, self.proposer.propose(runner, decodings, req_to_token))]
        # The verification reads its tokens to the host: no request keeps a device-selected token.
        runner.steps.release(slots)
        targets = verify(runner, decodings, chains, req_to_token)
        committed = [accept(c, t) for c, t in zip(chains, targets)]
        for d, c in zip(decodings, committed):
            self.proposer.committed(d.rid, d.tokens + c)
        return committed


def verify(runner, decodings: list[Decoding], chains, req_to_token) -> list[list[int]]:
    """The target's greedy token after every chain row, in calls of at most `rows` rows."""
    lengths = [len(c) for c in chains]
    cached = [d.cached for d in decodings]
    targets: list[list[int]] = [[] for _ in chains]
    for call in steps.plan(lengths, cached, int(runner.model.rows)):
        flat = np.concatenate([np.asarray(chains[r.seq][r.first : r.first + r.count], dtype=np.int32) for r in call])
        dev = runner.engine.HostTensor.from_dlpack(np.ascontiguousarray(flat)).to_hbm(runner.device)
        reqs, at = [], 0
        for r in call:
            blocks = runner.blocks(req_to_token, decodings[r.seq].slot, r.cached + r.count)
            reqs.append(runner.dec.Request([blocks], r.cached, dev[at : at + r.count], runner.dec.Keep.ALL))
            at += r.count
        host = np.asarray(runner.model.forward(reqs, runner.cache).to_host().numpy()).reshape(-1)
        at = 0
        for r in call:
            targets[r.seq] += [int(t) for t in host[at : at + r.count]]
            at += r.count
    return targets


def width_of(args) -> int:
    """The verification width SGLang's server arguments ask for: the draft-token count, or the
    draft steps plus the last token."""
    n = getattr(args, "speculative_num_draft_tokens", None)
    if n is None:
        n = int(getattr(args, "speculative_num_steps", None) or 3) + 1
    if int(n) < 2:
        raise ValueError("speculative_num_draft_tokens: a verification holds the last token and at least one draft")
    return int(n)


def ngram_of(args, width: int) -> Ngram:
    return Ngram(width - 1, int(getattr(args, "speculative_ngram_min_match_window_size", None) or 1),
                 int(getattr(args, "speculative_ngram_max_match_window_size", None) or 3))


def _record(**fields):
    """SGLang's verify input of the next step when SGLang is importable, else a plain record."""
    try:
        from sglang.srt.speculative.ngram_info import NgramVerifyInput
    except ImportError:
        import types

        return types.SimpleNamespace(**fields)
    return NgramVerifyInput(**fields)


def _pack(committed, width: int):
    import torch

    out = torch.zeros((len(committed), width), dtype=torch.int64)
    for row, tokens in zip(out, committed):
        row[: len(tokens)] = torch.tensor(tokens, dtype=torch.int64)
    return out.flatten()


def forward(runner, speculation: Speculation, batch, req_to_token, context: int):
    """One step of SGLang's speculative schedule: the result with the committed tokens."""
    import torch

    mode = batch.forward_mode
    if mode.is_extend():
        # A prompt step commits the target's next token; a request prefilled again has lost what
        # the proposer kept of it.
        speculation.proposer.forget(r.rid for r in batch.reqs)
        result = runner.issue(batch, req_to_token, overlap=False)
        result.read()
        committed = [(int(t),) for t in result.next_token_ids.tolist()]
        new_seq_lens = batch.seq_lens
    elif mode.is_decode():
        if not steps.greedy(batch):
            raise NotImplementedError("speculative verification selects greedy tokens; sampling reads scores")
        committed = speculation.decode(runner, batch, req_to_token, context)
        result = steps.result_class()((), len(committed))
        new_seq_lens = batch.seq_lens + torch.tensor([len(c) for c in committed], dtype=batch.seq_lens.dtype)
    else:
        raise ValueError(f"speculative decoding schedules no {mode} step")
    packed = _pack(committed, speculation.width)
    result.next_token_ids = packed
    result.accept_lens = torch.tensor([len(c) for c in committed], dtype=torch.int32)
    result.new_seq_lens = new_seq_lens
    result.speculative_num_draft_tokens = speculation.width
    result.next_draft_input = _record(draft_token_num=speculation.width, new_seq_lens=new_seq_lens,
                                      accept_tokens=packed, accept_lens=result.accept_lens)
    return result


_made: dict = {}


def worker_class():
    """SGLang's speculative worker over the plugin's target worker (`BaseSpecWorker` when SGLang is
    importable). SGLang builds it with the target worker; it drafts with the runner's proposer."""
    if "worker" in _made:
        return _made["worker"]
    try:
        from sglang.srt.speculative.base_spec_worker import BaseSpecWorker
    except ImportError:
        BaseSpecWorker = object

    class SpecWorker(BaseSpecWorker):
        _draft_worker = None  # SGLang reads it; the runner's proposer drafts instead

        def __init__(self, server_args, gpu_id, nccl_port, target_worker, *args, **kwargs):
            if BaseSpecWorker is not object:
                super().__init__()
            self.server_args = server_args
            self._target_worker = target_worker
            self.model_runner = target_worker.model_runner

        @property
        def target_worker(self):
            return self._target_worker

        @property
        def draft_worker(self):
            return None

        def forward_batch_generation(self, batch, *args, **kwargs):
            runner = self._target_worker.engine_runner
            if runner.speculation is None:
                raise RuntimeError("the runner loaded no proposer; the platform admits speculation first")
            return forward(runner, runner.speculation, batch, self._target_worker.request_table(),
                           int(self._target_worker.model_runner.model_config.context_len))

        def clear_cache_pool(self):
            runner = self._target_worker.engine_runner
            if runner.speculation is not None:
                runner.speculation.proposer.reset()

    _made["worker"] = SpecWorker
    return SpecWorker


def create_worker(_algorithm, _server_args=None):
    """SGLang's `SpeculativeAlgorithm.create_worker`, replaced: every admitted algorithm runs
    through the plugin's speculative worker."""
    return worker_class()
