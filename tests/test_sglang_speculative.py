"""The SGLang plugin's speculative decoding without a GPU: n-gram and draft-model proposers, the
greedy verification (the committed tokens are the greedy continuation whatever the drafts), the
result fields SGLang reads, platform refusals and the worker hook. The fake engine's greedy token is
a function of the row's input token and position (tests/test_sglang_steps.py)."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import sglang_fakes
from furiosa_opt_sglang import hooks, platform, speculative
from test_sglang_steps import Decoder, Mode, greedy_info, next_token, runner, table


def greedy_continuation(tokens, n):
    seq = list(tokens)
    for _ in range(n):
        seq.append(next_token(seq[-1], len(seq) - 1))
    return seq[len(tokens):]


def request(rid, prompt, output=()):
    return SimpleNamespace(rid=rid, origin_input_ids=list(prompt), output_ids=list(output))


def decode_batch(reqs, slots):
    seq_lens = [len(r.origin_input_ids) + len(r.output_ids) - 1 for r in reqs]
    return SimpleNamespace(forward_mode=Mode(False), reqs=reqs, req_pool_indices=torch.tensor(slots),
                           seq_lens=torch.tensor(seq_lens), input_ids=torch.tensor([0] * len(reqs)),
                           sampling_info=greedy_info(), return_logprob=False, decoding_reqs=None)


class Fixed:
    """A proposer that returns the drafts it was given, and records what it was told."""

    def __init__(self, drafts):
        self.drafts, self.commits, self.forgotten = drafts, [], []

    def propose(self, runner, decodings, req_to_token):
        return [list(self.drafts.get(d.rid, [])) for d in decodings]

    def committed(self, rid, tokens):
        self.commits.append((rid, tokens))

    def forget(self, rids):
        self.forgotten += list(rids)

    def reset(self):
        pass


def test_accept_keeps_drafts_while_they_match_the_target():
    assert speculative.accept((5, 1, 2, 3), [1, 2, 9, 4]) == (1, 2, 9)
    assert speculative.accept((5, 1, 2), [1, 2, 7]) == (1, 2, 7)  # every draft accepted: a bonus token
    assert speculative.accept((5, 8), [1, 2]) == (1,)
    assert speculative.accept((5,), [3]) == (3,)
    with pytest.raises(ValueError):
        speculative.accept((5, 1), [1])


def test_ngram_drafts_follow_the_latest_longest_earlier_match():
    ng = speculative.Ngram(k=3, min_n=1, max_n=3)
    assert ng.draft([1, 2, 3, 4, 1, 2], 3) == [3, 4, 1]  # [1, 2] occurred at 0
    assert ng.draft([7, 1, 2, 9, 1, 2, 5, 1, 2], 3) == [5, 1, 2]  # the latest occurrence wins
    assert ng.draft([4, 5, 6, 9, 5, 6, 8, 4, 5, 6], 2) == [9, 5]  # [4, 5, 6] beats the later [5, 6]
    assert ng.draft([1, 2, 3], 3) == []
    assert ng.draft([1, 1], 2) == [1]  # drafts stop at the end of the known tokens
    assert ng.draft([1, 2, 1], 0) == []
    with pytest.raises(ValueError):
        speculative.Ngram(k=0)


def test_verification_commits_the_greedy_continuation():
    r = runner()
    reqs = [request("a", [3, 4, 5]), request("b", [9, 8], [7]), request("c", [1, 2, 3, 4])]
    good = greedy_continuation([3, 4, 5], 3)
    drafts = {"a": good[:3], "b": [0, 0], "c": greedy_continuation([1, 2, 3, 4], 2)[:1] + [999]}
    spec = speculative.Speculation(Fixed(drafts), width=4)
    t = table()
    result = speculative.forward(r, spec, decode_batch(reqs, [0, 1, 2]), t, context=64)
    want = {"a": greedy_continuation([3, 4, 5], 4), "b": greedy_continuation([9, 8, 7], 1),
            "c": greedy_continuation([1, 2, 3, 4], 2)}
    assert result.accept_lens.tolist() == [4, 1, 2]
    packed = result.next_token_ids.view(3, 4)
    for i, rid in enumerate("abc"):
        assert packed[i, : len(want[rid])].tolist() == want[rid]
    assert result.new_seq_lens.tolist() == [2 + 4, 2 + 1, 3 + 2]
    assert result.speculative_num_draft_tokens == 4
    assert result.next_draft_input.accept_lens.tolist() == [4, 1, 2]
    # Every chain row is kept, in calls of at most `rows` rows, at the request's own positions.
    rows = [sum(len(tokens) for _, _, tokens, _ in call) for call in r.model.calls]
    assert max(rows) <= Decoder.rows and sum(rows) == 4 + 3 + 3
    assert all(keep == "all" for call in r.model.calls for *_, keep in call)
    assert r.model.calls[0][0][1] == 2  # request a caches its 2 tokens before the last
    assert spec.proposer.commits[0] == ("a", (3, 4, 5, *want["a"]))


def test_context_end_limits_the_drafts():
    r = runner()
    spec = speculative.Speculation(Fixed({"a": [1, 2, 3]}), width=4)
    reqs = [request("a", list(range(10, 20)))]
    result = speculative.forward(r, spec, decode_batch(reqs, [0]), table(), context=11)
    assert result.accept_lens.tolist() == [1]  # 9 cached of 11: room for the last token and one draft
    assert len(r.model.calls[0][0][2]) == 2


def test_ngram_speculation_matches_plain_greedy_decoding():
    """Decode steps with n-gram drafts until 30 tokens are out: the same tokens as plain greedy
    decoding."""
    r = runner()
    spec = speculative.Speculation(speculative.Ngram(k=3), width=4)
    req = request("a", [2, 2, 2, 2, 2])
    steps_taken = 0
    while len(req.output_ids) < 30:
        result = speculative.forward(r, spec, decode_batch([req], [0]), table(context=128), context=128)
        n = int(result.accept_lens[0])
        req.output_ids += result.next_token_ids[:n].tolist()
        steps_taken += 1
    assert req.output_ids[:30] == greedy_continuation([2, 2, 2, 2, 2], 30)
    assert steps_taken <= 30


class DraftDecoder(Decoder):
    """A draft model whose greedy token agrees with the target's except after the token `wrong`."""

    def __init__(self, wrong=None):
        super().__init__()
        self.wrong = wrong

    def forward(self, reqs, cache):
        out = super().forward(reqs, cache)
        if self.wrong is not None:
            vals = out.values.copy()
            last = [int(r.tokens.values.tolist()[-1]) for r in reqs if r.keep == "last"]
            for i, t in enumerate(last):
                if t == self.wrong:
                    vals[i] = (vals[i] + 1) % 1000
            out = type(out)(vals)
        return out


def test_draft_model_feeds_each_token_once_and_drops_rejected_rows():
    r = runner()
    draft = DraftDecoder()
    spec = speculative.Speculation(speculative.DraftModel(draft, None, k=3), width=4)
    req = request("a", [5, 6, 7])
    result = speculative.forward(r, spec, decode_batch([req], [0]), table(), context=64)
    want = greedy_continuation([5, 6, 7], 4)
    assert result.next_token_ids[:4].tolist() == want  # a perfect draft: all accepted plus a bonus
    # The draft fed the prompt once, then one row per further draft.
    fed = [(cached, tokens) for call in draft.calls for _, cached, tokens, _ in call]
    assert fed == [(0, [5, 6, 7]), (3, [want[0]]), (4, [want[1]])]
    req.output_ids += want
    draft.calls.clear()
    speculative.forward(r, spec, decode_batch([req], [0]), table(), context=64)
    # Next step: the draft holds 5 of the 7 tokens (its rows of d1, d2 match the commit).
    assert [(c, t) for call in draft.calls for _, c, t, _ in call][0] == (5, [want[2], want[3]])


def test_a_wrong_draft_model_still_commits_the_greedy_tokens():
    r = runner()
    prompt = [5, 6, 7]
    wrong = greedy_continuation(prompt, 1)[0]  # the draft errs after the first new token
    draft = DraftDecoder(wrong=wrong)
    spec = speculative.Speculation(speculative.DraftModel(draft, None, k=3), width=4)
    req = request("a", prompt)
    out = []
    while len(out) < 12:
        result = speculative.forward(r, spec, decode_batch([req], [0]), table(), context=64)
        n = int(result.accept_lens[0])
        got = result.next_token_ids[:n].tolist()
        out += got
        req.output_ids += got
    assert out[:12] == greedy_continuation(prompt, 12)
    held = spec.proposer.held["a"]
    assert held == tuple(prompt + out)[: len(held)]  # what the draft holds is the committed history


def test_prompt_steps_commit_one_token_and_forget_the_proposer(monkeypatch):
    r = runner()
    fixed = Fixed({})
    spec = speculative.Speculation(fixed, width=3)
    reqs = [request("a", [1, 2, 3]), request("b", [4, 5])]
    b = SimpleNamespace(forward_mode=Mode(True), reqs=reqs, req_pool_indices=torch.tensor([0, 1]),
                        seq_lens=torch.tensor([3, 2]), extend_lens=[3, 2], input_ids=torch.tensor([1, 2, 3, 4, 5]),
                        decoding_reqs=None, sampling_info=greedy_info(), return_logprob=False)
    result = speculative.forward(r, spec, b, table(), context=64)
    assert result.accept_lens.tolist() == [1, 1]
    assert result.next_token_ids.view(2, 3)[:, 0].tolist() == [next_token(3, 2), next_token(5, 1)]
    assert result.new_seq_lens.tolist() == [3, 2]
    assert fixed.forgotten == ["a", "b"]


def test_platform_admits_ngram_and_draft_models_only():
    platform.check(speculative="NGRAM")
    platform.check(speculative="standalone", draft_model="/ckpt/draft")
    for kwargs, option in [(dict(speculative="EAGLE3"), "speculative_algorithm"),
                           (dict(speculative="STANDALONE"), "speculative_draft_model_path"),
                           (dict(speculative="NGRAM", draft_topk=4), "speculative_eagle_topk")]:
        with pytest.raises(platform.Refused) as e:
            platform.check(**kwargs)
        assert e.value.option == option
    args = SimpleNamespace(speculative_num_draft_tokens=None, speculative_num_steps=4)
    assert speculative.width_of(args) == 5
    with pytest.raises(ValueError):
        speculative.width_of(SimpleNamespace(speculative_num_draft_tokens=1))


def test_spec_worker_hook_routes_to_the_engine(monkeypatch):
    sglang_fakes.install(monkeypatch)
    assert hooks.register() == len(hooks.HOOKS)
    made = {t: f for t, f, _ in sglang_fakes.HookRegistry.installed}
    cls = made["sglang.srt.speculative.spec_info.SpeculativeAlgorithm.create_worker"]("NGRAM", None)
    assert issubclass(cls, sglang_fakes.BaseSpecWorker)
    r = runner()
    r.speculation = speculative.Speculation(speculative.Ngram(k=2), width=3)
    t = table()
    target = SimpleNamespace(engine_runner=r, request_table=lambda: t,
                             model_runner=SimpleNamespace(model_config=SimpleNamespace(context_len=64)))
    w = cls(SimpleNamespace(), 0, 0, target)
    assert w.target_worker is target and w.draft_worker is None
    result = w.forward_batch_generation(decode_batch([request("a", [1, 2, 1, 2])], [0]))
    assert isinstance(result.next_draft_input, sglang_fakes.NgramVerifyInput)
    n = int(result.accept_lens[0])
    assert result.next_token_ids[:n].tolist() == greedy_continuation([1, 2, 1, 2], n)
    w.clear_cache_pool()
