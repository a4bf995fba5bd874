"""Overlap-scheduled generation steps: SGLang's scheduled batches run through the engine without a
host round trip between steps.

SGLang's overlap scheduler issues step n+1 before it processes step n's result. A greedy step
here returns once its engine calls are submitted: the selected tokens stay on the device, each
request's next decode row reads its input token from there (an engine request may take its tokens
from any device tensor), and the scheduler hook `collect` reads them (one device-to-host copy per
engine call) just before SGLang processes the step. Steps that need scores (sampling, logprobs,
penalties, grammars, logit bias) are refused: the engine's decoder calls return tokens, not logits.
The reference's contract: integrations/furiosa-opt-sglang/furiosa_opt_sglang/generation/__init__.py
(`issue`, `Sampled`, `device_argmax`) and generation/sequence.py (calls of at most `rows` rows).

Nothing here imports SGLang at module load: the result class subclasses SGLang's
`GenerationBatchResult` when SGLang is importable, and a plain record with the same fields otherwise.
"""

from __future__ import annotations

import dataclasses
from collections import deque

import numpy as np


@dataclasses.dataclass(frozen=True)
class Run:
    """A request's rows in one engine call: batch index, positions cached before the run, offset of
    the run in the request's new tokens, its row count, and whether it ends the request's rows."""

    seq: int
    cached: int
    first: int
    count: int
    last: bool


def plan(lengths: list[int], cached: list[int], rows: int) -> list[list[Run]]:
    """Splits the batch's new rows, in batch order, into engine calls of at most `rows` rows; a
    request whose rows straddle two calls continues in the next one after its earlier runs."""
    if rows <= 0:
        raise ValueError("a decoder call holds at least one row")
    calls: list[list[Run]] = [[]]
    room = rows
    for i, (n, c) in enumerate(zip(lengths, cached)):
        if n <= 0:
            raise ValueError(f"request {i} schedules {n} rows")
        done = 0
        while done < n:
            if room == 0:
                calls.append([])
                room = rows
            take = min(room, n - done)
            calls[-1].append(Run(i, c + done, done, take, done + take == n))
            done += take
            room -= take
    return [c for c in calls if c]


def greedy(batch) -> bool:
    """Whether the device's first-maximum argmax selects the tokens SGLang's sampler would: every
    request greedy, no logprobs, penalties, grammar, logit bias or custom logit processor."""
    info = batch.sampling_info
    return bool(
        getattr(info, "is_all_greedy", False)
        and not getattr(batch, "return_logprob", False)
        and not getattr(info, "grammars", None)
        and getattr(info, "logit_bias", None) is None
        and getattr(info, "acc_additive_penalties", None) is None
        and getattr(info, "acc_scaling_penalties", None) is None
        and not getattr(info, "has_custom_logit_processor", False)
    )


class _Record:
    """The fields of SGLang's GenerationBatchResult the scheduler reads, when SGLang is absent."""

    def __init__(self, logits_output=None, next_token_ids=None, can_run_cuda_graph=False):
        self.logits_output = logits_output
        self.next_token_ids = next_token_ids
        self.can_run_cuda_graph = can_run_cuda_graph


_classes: dict = {}


def result_class():
    """The step result class: a subclass of SGLang's GenerationBatchResult (or of `_Record`)."""
    try:
        from sglang.srt.layers.logits_processor import LogitsProcessorOutput
        from sglang.srt.managers.utils import GenerationBatchResult
    except ImportError:
        GenerationBatchResult, LogitsProcessorOutput = _Record, None
    key = (GenerationBatchResult, LogitsProcessorOutput)
    if key in _classes:
        return _classes[key]

    class Sampled(GenerationBatchResult):
        """A greedy step whose tokens stay on the device until `collect` (once, before SGLang
        processes the step). Until then `next_token_ids` holds zeros, which SGLang relays as the
        next decode rows' inputs; those rows read the device tokens instead."""

        def __init__(self, calls: list, size: int):
            import torch

            logits = LogitsProcessorOutput(next_token_logits=None) if LogitsProcessorOutput is not None else None
            super().__init__(logits_output=logits, next_token_ids=torch.zeros(size, dtype=torch.int64),
                             can_run_cuda_graph=False)
            self.calls = calls  # [(batch indices of the kept rows, the call's device tokens)]
            self.size = size

        def collect(self) -> None:
            import torch

            if not self.calls:
                return
            ids = torch.zeros(self.size, dtype=torch.int64)
            for kept, tokens in self.calls:
                host = np.asarray(tokens.to_host().numpy()).reshape(-1)[: len(kept)]
                ids[torch.tensor(kept, dtype=torch.int64)] = torch.from_numpy(host.astype(np.int64))
            self.next_token_ids = ids
            self.calls = []

    _classes[key] = Sampled
    return Sampled


class State:
    """A runner's step bookkeeping: the results issued and not yet certainly processed (oldest
    first), and each request-pool row's next input token while a greedy step holds it on the device
    (the call's token tensor and the row in it)."""

    def __init__(self):
        self.issued: deque = deque()
        self.selected: dict[int, tuple] = {}

    def release(self, slots) -> None:
        """Drops the device tokens of freed request-pool rows (their requests run no further step)."""
        for s in slots:
            self.selected.pop(int(s), None)


def _ints(x) -> list[int]:
    if hasattr(x, "tolist"):
        return [int(v) for v in x.tolist()]
    return [int(v) for v in x]


def issue(runner, batch, req_to_token, *, overlap: bool):
    """Submits a scheduled generation batch's engine calls and returns its `Sampled` result without
    waiting for them. With `overlap`, SGLang processes the previous step while the device runs
    this one; either way a step must be collected before the second step after it is issued."""
    state: State = runner.steps
    while len(state.issued) > (1 if overlap else 0):
        old = state.issued.popleft()
        if old.calls:
            raise RuntimeError("SGLang processed a greedy step without collecting its tokens")
    mode = batch.forward_mode
    extend = mode.is_extend()
    if not (extend or mode.is_decode()):
        raise ValueError(f"unsupported forward mode {mode}")
    if not greedy(batch):
        raise NotImplementedError("sampling and scoring read scores the engine's calls do not return")
    slots = _ints(batch.req_pool_indices)
    seq_lens = _ints(batch.seq_lens)
    lengths = _ints(batch.extend_lens) if extend else [1] * len(slots)
    cached = [t - n for t, n in zip(seq_lens, lengths)]
    # Decode rows, and the decode requests a mixed extend batch carries, take the token the last
    # step left on the device; every other row reads the batch's uploaded IDs.
    running = {id(r) for r in (getattr(batch, "decoding_reqs", None) or ())}
    feed = {}
    for i, req in enumerate(batch.reqs):
        if (not extend or id(req) in running) and slots[i] in state.selected:
            feed[i] = state.selected[slots[i]]
    ids = np.asarray(_ints(batch.input_ids), dtype=np.int32)
    starts = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    if len(ids) != starts[-1]:
        raise ValueError(f"{len(ids)} input IDs for {starts[-1]} scheduled rows")
    calls = []
    for call in plan(lengths, cached, int(runner.model.rows)):
        host = [r for r in call if r.seq not in feed]
        uploaded = None
        if host:
            flat = np.concatenate([ids[starts[r.seq] + r.first : starts[r.seq] + r.first + r.count] for r in host])
            uploaded = runner.engine.HostTensor.from_dlpack(np.ascontiguousarray(flat)).to_hbm(runner.device)
        reqs, at, kept = [], 0, []
        for r in call:
            if r.seq in feed:
                src, row = feed[r.seq]
                tokens = src[row : row + 1]
            else:
                tokens = uploaded[at : at + r.count]
                at += r.count
            blocks = runner.blocks(req_to_token, slots[r.seq], r.cached + r.count)
            keep = runner.dec.Keep.LAST if r.last else runner.dec.Keep.NONE
            reqs.append(runner.dec.Request([blocks], r.cached, tokens, keep))
            if r.last:
                kept.append(r.seq)
        out = runner.model.forward(reqs, runner.cache)
        if kept:
            calls.append((kept, out))
            for row, i in enumerate(kept):
                state.selected[slots[i]] = (out, row)
        for r in call:
            if not r.last:  # a request's earlier runs keep nothing; a stale token must not feed it
                state.selected.pop(slots[r.seq], None)
    result = result_class()(calls, len(slots))
    state.issued.append(result)
    return result


def collect(_scheduler, _batch, result) -> None:
    """The hook before SGLang's `Scheduler.process_batch_result`: reads a step's device tokens."""
    if isinstance(result, result_class()):
        result.collect()
