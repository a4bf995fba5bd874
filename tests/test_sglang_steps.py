"""The SGLang plugin's scheduled steps, hooks, pools and host tier without a GPU: a fake engine
whose greedy token is a function of the row's input token and position, SGLang-shaped batches, and
stand-ins for the SGLang classes the plugin subclasses (tests/sglang_fakes.py)."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import sglang_fakes
from furiosa_opt_sglang import hicache, hooks, paging, platform, pools, steps
from furiosa_opt_sglang.runner import Runner

VOCAB = 1000


def next_token(token: int, position: int) -> int:
    return (7 * token + position + 1) % VOCAB


class Tensor:
    """A device tensor of the fake engine: values, plus how many uploads made it."""

    uploads = 0

    def __init__(self, values):
        self.values = np.asarray(values)

    def __getitem__(self, s):
        return Tensor(self.values[s])

    def to_hbm(self, device):
        Tensor.uploads += 1
        return self

    def to_host(self):
        return self

    def numpy(self):
        return self.values


class Decoder:
    rows = 4

    def __init__(self):
        self.calls = []

    def forward(self, reqs, cache):
        self.calls.append([(r.rows[0], r.cached, r.tokens.values.tolist(), r.keep) for r in reqs])
        out = []
        for r in reqs:
            t = r.tokens.values.tolist()
            if r.keep == "last":
                out.append(next_token(int(t[-1]), r.cached + len(t) - 1))
            elif r.keep == "all":
                out += [next_token(int(x), r.cached + i) for i, x in enumerate(t)]
        return Tensor(np.array(out, dtype=np.int32))


def runner():
    r = Runner.__new__(Runner)
    r.engine = SimpleNamespace(HostTensor=SimpleNamespace(from_dlpack=Tensor))
    r.dec = SimpleNamespace(Keep=SimpleNamespace(LAST="last", NONE="none", ALL="all"),
                            Request=lambda rows, cached, tokens, keep: SimpleNamespace(
                                rows=rows, cached=cached, tokens=tokens, keep=keep))
    r.model, r.device, r.cache = Decoder(), None, None
    r.steps = steps.State()
    return r


class Mode:
    def __init__(self, extend):
        self.extend = extend

    def is_extend(self):
        return self.extend

    def is_decode(self):
        return not self.extend


def greedy_info(**kw):
    return SimpleNamespace(is_all_greedy=True, grammars=None, logit_bias=None, acc_additive_penalties=None,
                           acc_scaling_penalties=None, has_custom_logit_processor=False, **kw)


def batch(reqs, slots, seq_lens, ids, extend_lens=None, decoding=None, info=None):
    return SimpleNamespace(forward_mode=Mode(extend_lens is not None), reqs=reqs,
                           req_pool_indices=torch.tensor(slots), seq_lens=torch.tensor(seq_lens),
                           extend_lens=extend_lens, input_ids=torch.tensor(ids), decoding_reqs=decoding,
                           sampling_info=info or greedy_info(), return_logprob=False)


def table(slots=4, context=64):
    t = np.zeros((slots, context), dtype=np.int64)
    for s in range(slots):
        t[s] = np.arange(context) + 16 * 8 * (s + 1)  # request s's pages start at block 8 (s + 1)
    return t


def expected(prompt, steps_):
    seq = list(prompt)
    for _ in range(steps_):
        seq.append(next_token(seq[-1], len(seq) - 1))
    return seq[len(prompt):]


def test_plan_splits_rows_into_calls_in_batch_order():
    calls = steps.plan([5, 1, 3], [0, 9, 2], 4)
    assert calls == [[steps.Run(0, 0, 0, 4, False)],
                     [steps.Run(0, 4, 4, 1, True), steps.Run(1, 9, 0, 1, True), steps.Run(2, 2, 0, 2, False)],
                     [steps.Run(2, 4, 2, 1, True)]]
    with pytest.raises(ValueError):
        steps.plan([0], [0], 4)


def test_overlap_steps_feed_decode_rows_from_the_device():
    """An extend step, then decode steps whose batch IDs are SGLang's relayed placeholders (zeros):
    each decode row reads the token the previous step left on the device, collected one step late
    as the overlap scheduler does."""
    r, tab = runner(), table()
    prompts = [[3, 1, 4, 1, 5, 9], [2, 7]]
    reqs = [object(), object()]
    first = r.issue(batch(reqs, [0, 2], [6, 2], prompts[0] + prompts[1], extend_lens=[6, 2]), tab)
    # Six rows at four a call: request 0 straddles two calls, request 1 rides the second.
    assert [len(c) for c in r.model.calls] == [1, 2]
    assert r.model.calls[0][0][3] == "none" and r.model.calls[1][0][3] == "last"
    assert torch.equal(first.next_token_ids, torch.zeros(2, dtype=torch.int64))
    got = [[], []]
    pending = first
    for i in range(4):
        lens = [6 + i + 1, 2 + i + 1]
        uploads = Tensor.uploads
        result = r.issue(batch(reqs, [0, 2], lens, [0, 0]), tab)
        assert Tensor.uploads == uploads  # both rows came from the device
        steps.collect(None, None, pending)  # SGLang processes the previous step now
        got = [g + [int(t)] for g, t in zip(got, pending.next_token_ids.tolist())]
        pending = result
    steps.collect(None, None, pending)
    got = [g + [int(t)] for g, t in zip(got, pending.next_token_ids.tolist())]
    assert got == [expected(p, 5) for p in prompts]
    # The decode calls read request 0's blocks from its table row (block 8 onwards).
    rows, cached, _, _ = r.model.calls[-1][0]
    assert rows == [8] and cached == 9


def test_a_step_left_uncollected_is_refused():
    r, tab = runner(), table()
    reqs = [object()]
    r.issue(batch(reqs, [1], [3], [5, 6, 7], extend_lens=[3]), tab)
    r.issue(batch(reqs, [1], [4], [0]), tab)
    with pytest.raises(RuntimeError, match="without collecting"):
        r.issue(batch(reqs, [1], [5], [0]), tab)


def test_without_overlap_each_step_is_processed_before_the_next():
    r, tab = runner(), table()
    reqs = [object()]
    s = r.issue(batch(reqs, [1], [3], [5, 6, 7], extend_lens=[3]), tab, overlap=False)
    with pytest.raises(RuntimeError, match="without collecting"):
        r.issue(batch(reqs, [1], [4], [0]), tab, overlap=False)
    s.collect()
    assert s.next_token_ids.tolist() == expected([5, 6, 7], 1)


def test_mixed_batch_feeds_only_running_decode_requests():
    """A mixed chunked-prefill batch: a new request's prompt rows are uploaded, the running
    request's one row comes from the device."""
    r, tab = runner(), table()
    old, new = object(), object()
    s = r.issue(batch([old], [0], [2], [4, 2], extend_lens=[2]), tab)
    s.collect()
    mixed = r.issue(batch([new, old], [1, 0], [3, 3], [1, 2, 3, 0], extend_lens=[3, 1], decoding=[old]), tab)
    mixed.collect()
    assert mixed.next_token_ids.tolist() == [expected([1, 2, 3], 1)[0], expected([4, 2], 2)[1]]


def test_scored_steps_are_refused():
    r, tab = runner(), table()
    b = batch([object()], [0], [2], [4, 2], extend_lens=[2], info=greedy_info())
    b.sampling_info.is_all_greedy = False
    with pytest.raises(NotImplementedError, match="scores"):
        r.issue(b, tab)
    b = batch([object()], [0], [2], [4, 2], extend_lens=[2])
    b.return_logprob = True
    with pytest.raises(NotImplementedError):
        r.issue(b, tab)


def test_freed_rows_drop_their_device_tokens():
    st = steps.State()
    st.selected = {1: ("t", 0), 2: ("t", 1)}
    st.release([1])
    assert list(st.selected) == [2]


def test_hooks_install_through_the_registry(monkeypatch):
    sglang_fakes.install(monkeypatch)
    assert hooks.register() == len(hooks.HOOKS)
    installed = {t: (f, k) for t, f, k in sglang_fakes.HookRegistry.installed}
    worker, kind = installed["sglang.srt.managers.tp_worker.TpModelWorker"]
    assert kind == "replace" and issubclass(worker, sglang_fakes.TpModelWorker)
    assert installed["sglang.srt.managers.scheduler.Scheduler.process_batch_result"] == (steps.collect, "before")
    assert installed["sglang.srt.mem_cache.allocation.assign_req_to_token_pool_func"][0] is paging.assign
    # Without a registry or SGLang nothing is installed.
    assert all(h.reason for h in hooks.HOOKS)


def test_worker_routes_scheduled_batches_to_the_engine(monkeypatch):
    sglang_fakes.install(monkeypatch)
    from furiosa_opt_sglang import worker

    r, tab = runner(), table()

    def bind(model_runner):
        model_runner.engine_runner = r
        model_runner.req_to_token_pool = SimpleNamespace(req_to_token=tab)

    monkeypatch.setattr(pools, "bind", bind)
    w = worker.worker_class()(SimpleNamespace(mem_fraction_static=0.8), gpu_id=0)
    assert w.enable_overlap
    res = w.forward_batch_generation(batch([object()], [0], [3], [5, 6, 7], extend_lens=[3]))
    assert isinstance(res, sglang_fakes.GenerationBatchResult)
    steps.collect(None, None, res)
    assert res.next_token_ids.tolist() == expected([5, 6, 7], 1)
    with pytest.raises(ValueError, match="ordinary"):
        w.forward_batch_generation(None)
    with pytest.raises(ValueError, match="ordinary"):
        w.forward_batch_generation(batch([object()], [0], [4], [0]), is_verify=True)


def test_request_pool_frees_device_tokens(monkeypatch):
    sglang_fakes.install(monkeypatch)
    st = steps.State()
    pool = pools.request_pool_class()(4, 32, st)
    st.selected = {0: ("t", 0), 3: ("t", 1)}
    pool.free_rows([3])
    assert list(st.selected) == [0] and 3 in pool.free_slots
    pool.clear()
    assert st.selected == {}


def test_pool_sizes():
    gib = 1 << 30
    s = pools.Sizes.plan(free_bytes=100 * gib, capacity_bytes=180 * gib, fraction=0.9, block_bytes=1 << 20, rows=256)
    # 100 GiB free less the 18 GiB outside the static fraction, in 1 MiB blocks, one dummy block.
    assert s.blocks == 82 * 1024 and s.tokens == (82 * 1024 - 1) * 16 and s.requests == 256
    s = pools.Sizes.plan(100 * gib, 180 * gib, 0.9, 1 << 20, 256, max_tokens=1000, max_requests=8)
    assert s.tokens == 992 and s.blocks == 63 and s.requests == 8
    with pytest.raises(ValueError, match="max_total_tokens"):
        pools.Sizes.plan(100 * gib, 180 * gib, 0.9, 1 << 20, 256, max_tokens=10**12)
    with pytest.raises(ValueError, match="mem_fraction_static"):
        pools.Sizes.plan(10 * gib, 180 * gib, 0.9, 1 << 20, 256)


def test_assign_writes_each_requests_slots():
    t = torch.zeros(3, 8, dtype=torch.int64)
    paging.assign(torch.tensor([2, 0]), t, torch.tensor([1, 0]), torch.tensor([3, 2]),
                  torch.tensor([10, 11, 20, 21]), 2)
    assert t[2, 1:3].tolist() == [10, 11] and t[0, 0:2].tolist() == [20, 21]


def test_requests_with_unserved_inputs_are_refused():
    with pytest.raises(platform.Refused) as e:
        platform.validate_request(None, SimpleNamespace(image_data=["x.png"]))
    assert e.value.option == "image_data"
    with pytest.raises(platform.Refused):
        platform.validate_request(None, SimpleNamespace(return_logprob=True))
    platform.validate_request(None, SimpleNamespace(text="hi"))


def test_host_tier_pages_and_runs():
    assert hicache.pages(torch.arange(32, 64)) == [2, 3]
    with pytest.raises(ValueError, match="whole pages"):
        hicache.pages(torch.arange(0, 8))
    with pytest.raises(ValueError, match="consecutive"):
        hicache.pages(torch.arange(8, 24))
    assert hicache.runs([4, 5, 6, 9, 10], [0, 1, 7, 8, 9]) == [(4, 0, 2), (6, 7, 1), (9, 8, 2)]


class _Copy:
    def __init__(self, log, what, fail=False):
        self.log, self.what, self.fail = log, what, fail

    def wait(self):
        self.log.append(("waited", self.what))
        if self.fail:
            raise RuntimeError("copy failed")


class _Buffer:
    def __init__(self, log, name, fail_on=None):
        self.log, self.name, self.fail_on = log, name, fail_on

    def slice(self, offset, size):
        return SimpleNamespace(
            to_host=lambda host: self._copy(("d2h", self.name, offset, size, host.where)),
            to_hbm=lambda dev: self._copy(("h2d", self.name, offset, size, dev.where)),
            where=(self.name, offset, size))

    def _copy(self, what):
        self.log.append(what)
        return _Copy(self.log, what, fail=self.fail_on is not None and self.fail_on in what)


def test_host_tier_copies_pages_and_poisons_on_failure():
    log = []
    storage = SimpleNamespace(spec=SimpleNamespace(pools=[SimpleNamespace(bytes=100)]), blocks=64,
                              layers=[_Buffer(log, "L0"), _Buffer(log, "L1", fail_on="L1")])
    engine = SimpleNamespace(HostBuffer=lambda n: _Buffer(log, "host"))
    tier = hicache.HostTier(engine, storage, pages=8)
    tier.backup(torch.arange(16 * 4, 16 * 6), torch.arange(16 * 2, 16 * 4))  # blocks 4,5 -> pages 2,3
    assert ("d2h", "L0", 400, 200, ("host", 200, 200)) in log
    with pytest.raises(RuntimeError, match="poisoned"):
        tier.wait()
    # Both copies were waited for before the failure was raised.
    assert sum(1 for e in log if e[0] == "waited") == 2
    with pytest.raises(RuntimeError, match="poisoned"):
        tier.load(torch.arange(32, 48), torch.arange(64, 80), 0)
    with pytest.raises(ValueError, match="out of range"):
        hicache.HostTier(engine, storage, pages=1).backup(torch.arange(16), torch.arange(16, 32))


def test_host_pool_class_adapts_the_tier(monkeypatch):
    sglang_fakes.install(monkeypatch)
    log = []
    storage = SimpleNamespace(spec=SimpleNamespace(pools=[SimpleNamespace(bytes=100)]), blocks=64,
                              layers=[_Buffer(log, "L0"), _Buffer(log, "L1")])
    monkeypatch.setitem(__import__("sys").modules, "furiosa_opt_engine",
                        SimpleNamespace(HostBuffer=lambda n: _Buffer(log, "host")))
    device_pool = SimpleNamespace(storage=storage, size=64 * 16, dtype=torch.bfloat16)
    host = hicache.host_pool_class()(device_pool, 2.0, 0, 16)
    assert host.tier.pages == 128
    host.load_to_device_per_layer(device_pool, torch.arange(16), torch.arange(16, 32), 1, "kernel")
    assert log[-1] == ("h2d", "host", 0, 100, ("L1", 100, 100))
    with pytest.raises(ValueError):
        hicache.host_pool_class()(device_pool, 2.0, 0, 32)


def test_model_override_args_replace_config_keys(tmp_path):
    import json

    (tmp_path / "config.json").write_text(json.dumps({"architectures": ["Qwen3ForCausalLM"], "rope_theta": 1e6}))
    assert pools.overridden(str(tmp_path), None) is None
    assert pools.overridden(str(tmp_path), "{}") is None
    got = pools.overridden(str(tmp_path), '{"rope_scaling": {"rope_type": "linear", "factor": 2.0}}')
    assert got == {"architectures": ["Qwen3ForCausalLM"], "rope_theta": 1e6,
                   "rope_scaling": {"rope_type": "linear", "factor": 2.0}}
    with pytest.raises(ValueError, match="json_model_override_args"):
        pools.overridden(str(tmp_path), "[1, 2]")
