"""Speculative decoding in the vLLM plugin without a GPU: the runner feeds drafts after the newest
token, keeps every row, accepts drafts while they match the target's greedy tokens, and the
output equals plain greedy decoding whatever the drafts (a fake engine whose greedy token depends
on the fed token)."""

from types import SimpleNamespace

import numpy as np
import pytest

from furiosa_opt_vllm import admission, speculation
from furiosa_opt_vllm.runner import Runner


def test_accept():
    assert speculation.accept([], [7]) == [7]
    assert speculation.accept([5, 6], [5, 6, 9]) == [5, 6, 9]  # all accepted, plus the bonus token
    assert speculation.accept([5, 1], [5, 6, 9]) == [5, 6]
    assert speculation.accept([4, 6], [5, 6, 9]) == [5]
    with pytest.raises(ValueError):
        speculation.accept([1, 2], [1, 2])


def test_admission_serves_ngram_and_draft_models():
    admission.options(pipeline=1, tensor=1, speculative="ngram", lora=False, kv_cache_dtype="auto")
    admission.options(pipeline=1, tensor=1, speculative="draft_model", lora=False, kv_cache_dtype="auto")
    with pytest.raises(admission.Refused, match="one GPU a replica"):
        admission.options(pipeline=1, tensor=2, speculative="draft_model", lora=False, kv_cache_dtype="auto")
    for method in ("eagle", "mtp", "suffix"):
        with pytest.raises(admission.Refused, match="n-gram prompt lookup"):
            admission.options(pipeline=1, tensor=1, speculative=method, lora=False, kv_cache_dtype="auto")


def nxt(token: int) -> int:
    return (token * 7 + 3) % 50


class FakeTensor:
    def __init__(self, a):
        self.a = np.asarray(a, dtype=np.int32)

    def __getitem__(self, s):
        return FakeTensor(self.a[s])

    def to_hbm(self, device):
        return self

    def to_host(self):
        return self

    def numpy(self):
        return self.a


class FakeModel:
    """Greedy token after each kept row: a function of that row's token."""

    rows = 8192  # rows a call takes

    def __init__(self, keep):
        self.keep = keep
        self.calls = []

    def forward(self, reqs, cache, adapters=None):
        out = []
        for r in reqs:
            toks = r.tokens.a.tolist()
            self.calls.append((r.cached, toks, r.keep))
            if r.keep == self.keep.ALL:
                out += [nxt(t) for t in toks]
            elif r.keep == self.keep.LAST:
                out.append(nxt(toks[-1]))
        return FakeTensor(out)


def make_runner():
    keep = SimpleNamespace(NONE="none", LAST="last", ALL="all")
    model = FakeModel(keep)
    r = Runner(model, device=None, cache=None)
    r.engine = SimpleNamespace(HostTensor=SimpleNamespace(from_dlpack=FakeTensor))
    r.dec = SimpleNamespace(Keep=keep, Request=lambda rows, cached, tokens, keep, adapter=None: SimpleNamespace(
        rows=rows, cached=cached, tokens=tokens, keep=keep, adapter=adapter))
    return r, model


def sched(new=(), cached=(), counts=None, spec=None):
    return SimpleNamespace(
        finished_req_ids=set(), scheduled_new_reqs=list(new),
        scheduled_cached_reqs=SimpleNamespace(req_ids=[c[0] for c in cached], new_block_ids=[None for _ in cached],
                                              num_computed_tokens=[c[1] for c in cached], resumed_req_ids=set(),
                                              all_token_ids={}),
        num_scheduled_tokens=counts, scheduled_spec_decode_tokens=spec or {})


@pytest.mark.parametrize("draft_kind", ["right", "wrong", "half", "none"])
def test_speculative_steps_equal_greedy_decoding(draft_kind):
    prompt = [3, 11, 4]
    greedy = []
    t = prompt[-1]
    for _ in range(12):
        t = nxt(t)
        greedy.append(t)

    r, model = make_runner()
    new = SimpleNamespace(req_id="a", prompt_token_ids=prompt, num_computed_tokens=0, block_ids=([0, 1],),
                          lora_request=None)
    ids, out = r.step(sched(new=[new], counts={"a": 3}))
    assert out == [[greedy[0]]]
    produced = list(out[0])
    computed = 3
    while len(produced) < 10:
        known = list(r.states["a"].tokens)
        if draft_kind == "right":
            d = [nxt(known[-1]), nxt(nxt(known[-1]))]
        elif draft_kind == "wrong":
            d = [(nxt(known[-1]) + 1) % 50, 0]
        elif draft_kind == "half":
            d = [nxt(known[-1]), (nxt(nxt(known[-1])) + 1) % 50]
        else:
            d = []
        n = 1 + len(d)
        ids, out = r.step(sched(cached=[("a", computed)], counts={"a": n}, spec={"a": d} if d else {}))
        got = out[0]
        assert got == greedy[len(produced):len(produced) + len(got)]
        expect = {"right": 3, "wrong": 1, "half": 2, "none": 1}[draft_kind]
        assert len(got) == expect
        # The call fed the newest token then the drafts, after the history, and kept every row.
        cached_at, fed, keep = model.calls[-1]
        assert cached_at == computed and fed == [known[-1]] + d
        assert keep == ("all" if d else "last")
        # vLLM rolls its computed positions back by the rejected drafts.
        computed += n - (len(d) - (len(got) - 1))
        produced += got
    assert produced == greedy[:len(produced)]
    assert r.states["a"].tokens == prompt + produced


def test_drafts_after_a_stale_history_are_refused():
    r, _ = make_runner()
    new = SimpleNamespace(req_id="a", prompt_token_ids=[1, 2, 3], num_computed_tokens=0, block_ids=([0],),
                          lora_request=None)
    r.step(sched(new=[new], counts={"a": 2}))  # a prompt chunk: nothing sampled
    with pytest.raises(ValueError, match="drafts scheduled before the newest token"):
        r.step(sched(cached=[("a", 1)], counts={"a": 2}, spec={"a": [5]}))


def test_draft_model_feeds_only_what_changed_and_output_stays_greedy():
    """The draft model's proposer on a host fake: its first call feeds the prompt, later calls feed
    the accepted tokens from the first difference with what it fed, each further draft one row;
    with the target verifying, the output is exactly the greedy continuation."""
    r, target = make_runner()
    draft_calls = []

    class FakeDraft(FakeModel):
        """Agrees with the target except after token 7 (so some drafts are rejected)."""

        cache = SimpleNamespace(pools=[SimpleNamespace(bytes=64)], groups=[SimpleNamespace(layers=[0])])

        def forward(self, reqs, cache, adapters=None):
            draft_calls.append([(q.cached, q.tokens.a.tolist()) for q in reqs])
            out = []
            for q in reqs:
                t = q.tokens.a.tolist()[-1]
                out.append((nxt(t) + (1 if t == 7 else 0)) % 50)
            return FakeTensor(out)

    r.dec.Cache = lambda spec, n: ("draft cache", n)
    cfg = SimpleNamespace(speculative_config=SimpleNamespace(num_speculative_tokens=3, model="draft"))
    prop = speculation.DraftModel(cfg, lambda path: FakeDraft(r.dec.Keep))
    prop.attach(r, 64)
    prompt = [3, 11, 4]
    new = SimpleNamespace(req_id="a", prompt_token_ids=prompt, num_computed_tokens=0, block_ids=([0, 1],),
                          lora_request=None)
    ids, out = r.step(sched(new=[new], counts={"a": 3}))
    drafts = prop.propose(ids, out, r)
    # The whole prompt and the first sampled token, then one row a further draft.
    assert draft_calls[0] == [(0, prompt + out[0])]
    assert [c[0][0] for c in draft_calls[1:]] == [4, 5]
    produced, computed = list(out[0]), 3
    greedy, t = [], prompt[-1]
    for _ in range(20):
        t = nxt(t)
        greedy.append(t)
    while len(produced) < 12:
        d = drafts[0]
        n = 1 + len(d)
        before = len(draft_calls)
        ids, out = r.step(sched(cached=[("a", computed)], counts={"a": n}, spec={"a": d}))
        got = out[0]
        assert got == greedy[len(produced):len(produced) + len(got)]
        computed += n - (len(d) - (len(got) - 1))
        produced += got
        drafts = prop.propose(ids, out, r)
        # The first draft call starts at the first token the draft has not fed as known.
        first = draft_calls[before][0]
        assert first[0] <= len(r.states["a"].tokens) - 1
        assert first[1] == r.states["a"].tokens[first[0]:]
    assert produced == greedy[:len(produced)]
