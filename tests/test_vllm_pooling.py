"""Pooling in the vLLM plugin without a GPU: prompt chunks keep the rows their pooling needs
(LAST: the prompt's last row; MEAN: every row; CLS: the first chunk's rows), and the pooled row
goes through vLLM's embedding head (Matryoshka truncation, L2 normalization) or classification
head (softmax over the labels), with a fake engine whose hidden row is a function of the token."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from furiosa_opt_vllm import pooling
from furiosa_opt_vllm.runner import Runner

H = 6


def row(t: int) -> list[float]:
    return [float(t + j) * (1 if j % 2 else -1) for j in range(H)]


class FakeTensor:
    def __init__(self, a, dtype=np.int32):
        self.a = np.asarray(a, dtype=dtype)

    def __getitem__(self, s):
        return FakeTensor(self.a[s], self.a.dtype)

    def to_hbm(self, device):
        return self

    def to_host(self):
        return self

    def numpy(self):
        return self.a


class FakeModel:
    def __init__(self, keep):
        self.keep, self.calls = keep, []

    def forward(self, reqs, cache, adapters=None):
        out = []
        for r in reqs:
            toks = r.tokens.a.tolist()
            self.calls.append((r.cached, len(toks), r.keep))
            if r.keep == self.keep.ALL:
                out += [row(t) for t in toks]
            elif r.keep == self.keep.LAST:
                out.append(row(toks[-1]))
        return FakeTensor(np.array(out, dtype=np.float32).reshape(-1, H), np.float32)


def make_runner(task="embed", method="LAST", labels=0):
    keep = SimpleNamespace(NONE="none", LAST="last", ALL="all")
    model = FakeModel(keep)
    r = Runner(model, device=None, cache=None, pooling_config={"task": task, "method": method, "labels": labels})
    r.engine = SimpleNamespace(HostTensor=SimpleNamespace(from_dlpack=FakeTensor))
    r.dec = SimpleNamespace(Keep=keep, Request=lambda rows, cached, tokens, keep, adapter=None: SimpleNamespace(
        rows=rows, cached=cached, tokens=tokens, keep=keep))
    return r, model


def sched(new=(), cached=(), counts=None):
    return SimpleNamespace(
        finished_req_ids=set(), scheduled_new_reqs=list(new),
        scheduled_cached_reqs=SimpleNamespace(req_ids=[c[0] for c in cached], new_block_ids=[None for _ in cached],
                                              num_computed_tokens=[c[1] for c in cached], resumed_req_ids=set(),
                                              all_token_ids={}),
        num_scheduled_tokens=counts, scheduled_spec_decode_tokens={})


def run_chunks(r, prompt, chunks, params):
    new = SimpleNamespace(req_id="a", prompt_token_ids=prompt, num_computed_tokens=0, block_ids=([0, 1],),
                          lora_request=None, pooling_params=params)
    outs, at = [], 0
    for i, n in enumerate(chunks):
        so = sched(new=[new], counts={"a": n}) if i == 0 else sched(cached=[("a", at)], counts={"a": n})
        ids, sampled = r.step(so)
        assert sampled == [[]]
        outs.append(r.pooled[0])
        at += n
    return outs


@pytest.mark.parametrize("method", ["LAST", "MEAN", "CLS"])
def test_embedding_over_chunks(method):
    prompt = [3, 9, 4, 7, 1, 8, 2]
    r, model = make_runner("embed", method)
    outs = run_chunks(r, prompt, [3, 3, 1], SimpleNamespace(dimensions=None, use_activation=None))
    assert outs[0] is None and outs[1] is None and outs[2] is not None
    rows = torch.tensor([row(t) for t in prompt])
    want = {"LAST": rows[-1], "MEAN": rows.mean(0), "CLS": rows[0]}[method]
    assert torch.allclose(outs[2], torch.nn.functional.normalize(want, dim=-1), atol=1e-6)
    keeps = [k for _, _, k in model.calls]
    if method == "LAST":
        assert keeps == ["none", "none", "last"]
    elif method == "MEAN":
        assert keeps == ["all", "all", "last"]  # a one-row chunk keeps its row as LAST
    else:
        assert keeps == ["all", "none", "last"]


def test_matryoshka_dimensions_and_no_activation():
    r, _ = make_runner("embed", "LAST")
    (out,) = run_chunks(r, [5, 6], [2], SimpleNamespace(dimensions=3, use_activation=False))
    assert torch.allclose(out, torch.tensor(row(6)[:3]))


def test_classification_softmax_over_labels():
    r, _ = make_runner("classify", "LAST", labels=3)
    (out,) = run_chunks(r, [5, 6, 2], [3], SimpleNamespace(use_activation=None))
    assert torch.allclose(out, torch.softmax(torch.tensor(row(2)[:3]), -1))
    r, _ = make_runner("classify", "LAST", labels=1)
    (out,) = run_chunks(r, [4], [1], SimpleNamespace(use_activation=None))
    assert torch.allclose(out, torch.sigmoid(torch.tensor(row(4)[:1])))


def test_architectures_served_for_pooling():
    assert pooling.base_architecture("Qwen3ForCausalLM") == "Qwen3Model"
    assert pooling.base_architecture("Qwen3ForSequenceClassification") == "Qwen3ForSequenceClassification"
    assert pooling.base_architecture("MistralForCausalLM") is None
    with pytest.raises(pooling.Refused, match="pooling_type"):
        pooling.Pool(None, "STEP", 3)


def test_generation_requests_are_refused_by_a_pooling_model():
    r, _ = make_runner()
    new = SimpleNamespace(req_id="a", prompt_token_ids=[1, 2], num_computed_tokens=0, block_ids=([0],),
                          lora_request=None, pooling_params=None)
    with pytest.raises(ValueError, match="pooling requests only"):
        r.step(sched(new=[new], counts={"a": 2}))
