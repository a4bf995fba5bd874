"""The SGLang plugin's host contracts without a GPU: slots to engine blocks, batch parts from
SGLang's batch fields, server-argument refusals, entry points."""

import pickle

import pytest

from furiosa_opt_sglang import batch, paging, platform


def test_slots_map_to_blocks_page_by_page():
    slots = list(range(32, 64)) + list(range(160, 176))
    assert paging.blocks(slots, 40) == [2, 3, 10]
    with pytest.raises(paging.Misaligned):
        paging.blocks([5] * 16, 1)


def test_extend_parts_follow_batch_order():
    parts = batch.parts([3, 1], [20, 7], [4, 0], [16, 7])
    assert parts == [batch.Part(3, 4, 0, 16, True), batch.Part(1, 0, 16, 7, True)]
    with pytest.raises(ValueError):
        batch.parts([0], [10], [4], [5])
    assert batch.decode_parts([5, 6], [9, 1]) == [batch.Part(5, 8, 0, 1, True), batch.Part(6, 0, 1, 1, True)]


def test_request_blocks_cover_history_and_new_tokens():
    table = {0: list(range(16, 64))}
    assert batch.request_blocks(table, batch.Part(0, 20, 0, 5, True)) == [1, 2]


@pytest.mark.parametrize(("kwargs", "option"), [(dict(pp_size=2), "pp_size"), (dict(tp_size=6), "tp_size"),
                                                (dict(page_size=1), "page_size"),
                                                (dict(speculative="EAGLE"), "speculative_algorithm"),
                                                (dict(lora=True), "enable_lora"),
                                                (dict(kv_cache_dtype="fp8_e4m3"), "kv_cache_dtype")])
def test_refusals_name_the_option(kwargs, option):
    with pytest.raises(platform.Refused) as e:
        platform.check(**kwargs)
    assert e.value.option == option
    assert pickle.loads(pickle.dumps(e.value)).option == option
    platform.check(tp_size=8)


def test_entry_points():
    import furiosa_opt_sglang

    assert furiosa_opt_sglang.activate() == "furiosa_opt_sglang.platform.Platform"
    furiosa_opt_sglang.register()


def test_runner_embeds_the_last_rows():
    """An embedding batch keeps each request's last row and L2-normalizes it (a fake engine whose
    hidden row is a function of the token)."""
    from types import SimpleNamespace

    import numpy as np
    import torch

    from furiosa_opt_sglang.runner import Runner

    class T:
        def __init__(self, a):
            self.a = np.asarray(a)

        def __getitem__(self, s):
            return T(self.a[s])

        def to_hbm(self, device):
            return self

        def to_host(self):
            return self

        def numpy(self):
            return self.a

    keep = SimpleNamespace(LAST="last", NONE="none")
    out = SimpleNamespace(HIDDEN="hidden", TOKENS="tokens")
    seen = []

    class Model:
        output = "hidden"

        def forward(self, reqs, cache):
            seen.extend((r.cached, r.tokens.a.tolist(), r.keep) for r in reqs)
            return T(np.array([[float(r.tokens.a[-1]), 1.0, -2.0] for r in reqs], dtype=np.float32))

    r = Runner.__new__(Runner)
    r.engine = SimpleNamespace(HostTensor=SimpleNamespace(from_dlpack=T))
    r.dec = SimpleNamespace(Keep=keep, Output=out, Request=lambda rows, cached, tokens, keep: SimpleNamespace(
        rows=rows, cached=cached, tokens=tokens, keep=keep))
    r.model, r.device, r.cache = Model(), None, None
    table = [list(range(0, 64)), list(range(64, 128))]
    got = r.embed([0, 1], [3, 2], [0, 0], [3, 2], [4, 5, 6, 7, 8], table)
    want = torch.nn.functional.normalize(torch.tensor([[6.0, 1.0, -2.0], [8.0, 1.0, -2.0]]), dim=-1)
    assert torch.allclose(got, want)
    assert seen == [(0, [4, 5, 6], "last"), (0, [7, 8], "last")]
    raw = r.embed([0], [3], [0], [3], [4, 5, 6], table, normalize=False)
    assert torch.allclose(raw, torch.tensor([[6.0, 1.0, -2.0]]))
    Model.output = "tokens"
    with pytest.raises(ValueError, match="hidden rows"):
        r.embed([0], [3], [0], [3], [4, 5, 6], table)
