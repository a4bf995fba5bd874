"""Overlap-scheduled generation steps: SGLang's scheduled batches run through the engine without a
host round trip between steps.

SGLang's overlap scheduler issues step n+1 before it processes step n's result. A greedy step
here returns once its engine calls are submitted: the selected tokens stay on the device, each
request's next decode row reads its input token from there (an engine request may take its tokens
from any device tensor), and the scheduler hook `collect` reads them (one device-to-host copy per
engine call) just before SGLang processes the step. Issued steps are numbered: step n is refused
while step n - 2 (overlap) or n - 1 (synchronous schedule) is still unread, which is SGLang's
contract broken. Steps that need scores (sampling, logprobs,
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
    """The step result class, `DeviceStep`: a subclass of SGLang's GenerationBatchResult (of
    `_Record` without SGLang)."""
    try:
        from sglang.srt.layers.logits_processor import LogitsProcessorOutput
        from sglang.srt.managers.utils import GenerationBatchResult
    except ImportError:
        GenerationBatchResult, LogitsProcessorOutput = _Record, None
    key = (GenerationBatchResult, LogitsProcessorOutput)
    if key in _classes:
        return _classes[key]

    class DeviceStep(GenerationBatchResult):
        """A step's selected tokens while they are still on the device. `reads` pairs the batch
        indices of each engine call's kept rows with the call's output tensor; `read()` copies them
        to the host once and puts them in `next_token_ids`, which until then holds zeros (SGLang
        relays those as the next decode rows' inputs, and those rows take the device tokens)."""

        def __init__(self, reads, size: int, number: int = -1):
            import torch

            logits = LogitsProcessorOutput(next_token_logits=None) if LogitsProcessorOutput is not None else None
            super().__init__(logits_output=logits, next_token_ids=torch.zeros(size, dtype=torch.int64),
                             can_run_cuda_graph=False)
            self.reads = list(reads)
            self.size, self.number = size, number

        @property
        def unread(self) -> bool:
            return bool(self.reads)

        def read(self) -> None:
            import torch

            if not self.reads:
                return
            host = np.zeros(self.size, dtype=np.int64)
            for where, tokens in self.reads:
                host[where] = np.asarray(tokens.to_host().numpy()).reshape(-1)[: len(where)]
            self.next_token_ids = torch.from_numpy(host)
            self.reads = []

        collect = read  # the name SGLang-facing code calls

    _classes[key] = DeviceStep
    return DeviceStep


class State:
    """A runner's step bookkeeping: a count of the steps issued, the results not yet read (by step
    number), and each request-pool row's next input token while a step keeps it on the device
    (the call's output tensor and the row in it)."""

    def __init__(self):
        self.issued_steps = 0
        self.unread: dict[int, object] = {}
        self.selected: dict[int, tuple] = {}

    def release(self, slots) -> None:
        """Drops the device tokens of freed request-pool rows (their requests run no further step)."""
        for s in slots:
            self.selected.pop(int(s), None)

    def begin(self, lag: int) -> int:
        """The number of the step about to be issued. SGLang reads a step's result before it issues
        the step `lag + 1` after it (lag 1 under the overlap schedule, 0 without), so any older
        step still unread is an error."""
        n = self.issued_steps
        for k, step in list(self.unread.items()):
            if not step.unread:
                del self.unread[k]
            elif k < n - lag:
                raise RuntimeError(f"step {k} was issued and never read: SGLang issued step {n} "
                                   "without collecting its tokens")
        self.issued_steps = n + 1
        return n


def _ints(x) -> list[int]:
    if hasattr(x, "tolist"):
        return [int(v) for v in x.tolist()]
    return [int(v) for v in x]


def issue(runner, batch, req_to_token, *, overlap: bool):
    """Submits a scheduled generation batch's engine calls and returns its `DeviceStep` without
    waiting for them. With `overlap`, SGLang processes the previous step while the device runs this
    one; either way a step is read before the second step after it is issued."""
    state: State = runner.steps
    number = state.begin(1 if overlap else 0)
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
    # Decode rows, and the decode requests a mixed extend batch carries, take the token an earlier
    # step left on the device; every other row reads the batch's uploaded IDs.
    running = {id(r) for r in (getattr(batch, "decoding_reqs", None) or ())}
    from_device = {i: state.selected[slots[i]] for i, req in enumerate(batch.reqs)
                   if (not extend or id(req) in running) and slots[i] in state.selected}
    ids = np.asarray(_ints(batch.input_ids), dtype=np.int32)
    starts = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    if len(ids) != starts[-1]:
        raise ValueError(f"{len(ids)} input IDs for {starts[-1]} scheduled rows")
    reads = []
    for call in plan(lengths, cached, int(runner.model.rows)):
        uploaded_runs = [r for r in call if r.seq not in from_device]
        uploaded, offset = None, 0
        if uploaded_runs:
            flat = np.concatenate([ids[starts[r.seq] + r.first : starts[r.seq] + r.first + r.count]
                                   for r in uploaded_runs])
            uploaded = runner.engine.HostTensor.from_dlpack(np.ascontiguousarray(flat)).to_hbm(runner.device)
        requests, ends = [], []
        for r in call:
            if r.seq in from_device:
                src, row = from_device[r.seq]
                tokens = src[row : row + 1]
            else:
                tokens = uploaded[offset : offset + r.count]
                offset += r.count
            blocks = runner.blocks(req_to_token, slots[r.seq], r.cached + r.count)
            keep = runner.dec.Keep.LAST if r.last else runner.dec.Keep.NONE
            requests.append(runner.dec.Request([blocks], r.cached, tokens, keep))
            if r.last:
                ends.append(r.seq)
        out = runner.model.forward(requests, runner.cache)
        for r in call:
            if r.last:
                state.selected[slots[r.seq]] = (out, ends.index(r.seq))
            else:  # an earlier run of a request keeps nothing; its old device token must not feed it
                state.selected.pop(slots[r.seq], None)
        if ends:
            reads.append((np.asarray(ends, dtype=np.int64), out))
    result = result_class()(reads, len(slots), number)
    state.unread[number] = result
    return result


def collect(_scheduler, _batch, result) -> None:
    """The hook before SGLang's `Scheduler.process_batch_result`: reads a step's device tokens."""
    if isinstance(result, result_class()):
        result.read()
