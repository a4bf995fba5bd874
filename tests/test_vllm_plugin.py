"""The plugin's host contracts without a GPU: step planning, block tables, request state, the
runner's async collection on a host fake of the engine, refusals."""

import pytest

from furiosa_opt_vllm import admission, batch, paging
from furiosa_opt_vllm.request import State


def test_step_plan_slices_calls_to_the_decoder_rows():
    S = batch.Scheduled
    step = [S(0, 5, 5, batch.KEEP_LAST), S(10, 1, 0, batch.KEEP_LAST), S(3, 4, 4, batch.KEEP_NONE)]
    calls = batch.plan(step, rows=4)
    assert [[(r.seq, r.cached, r.offset, r.rows, r.keep, r.device) for r in c] for c in calls] == [
        [(0, 0, 0, 4, batch.KEEP_NONE, False)],
        [(0, 4, 4, 1, batch.KEEP_LAST, False), (1, 10, 0, 1, batch.KEEP_LAST, True),
         (2, 3, 0, 2, batch.KEEP_NONE, False)],
        [(2, 5, 2, 2, batch.KEEP_NONE, False)],
    ]
    assert all(sum(r.rows for r in c) <= 4 for c in calls)
    # Every row of a request with drafts comes back, whichever call holds it.
    every = batch.plan([S(0, 3, 3, batch.KEEP_ALL)], rows=2)
    assert [batch.kept_rows(r) for c in every for r in c] == [2, 1]
    # A request's known rows come before its device row, which is its last.
    mixed = batch.plan([S(7, 3, 2, batch.KEEP_LAST)], rows=8)[0]
    assert [(r.cached, r.rows, r.keep, r.device) for r in mixed] == [(7, 2, batch.KEEP_NONE, False),
                                                                      (9, 1, batch.KEEP_LAST, True)]


@pytest.mark.parametrize("bad", [batch.Scheduled(0, 0, 0, 0), batch.Scheduled(0, 3, 1, 1), batch.Scheduled(0, 2, 3, 1)])
def test_step_plan_refuses_bad_framing(bad):
    with pytest.raises(batch.Framing):
        batch.plan([bad], rows=8)


class _FakeTensor:
    def __init__(self, values):
        self.values = list(values)

    def __getitem__(self, sl):
        return _FakeTensor(self.values[sl])

    def numpy(self):
        import numpy as np

        return np.asarray(self.values, dtype=np.int32)

    def to_host(self):
        self.reads += 1
        return self

    reads = 0


class _FakeEngine:
    """Decoder calls on the host: each kept row's token is (its input token + 1)."""

    class HostTensor:
        @staticmethod
        def from_dlpack(a):
            return _FakeHost(a)

    def __init__(self, rows):
        from types import SimpleNamespace

        self.rows = rows
        self.calls = []
        self.dec = SimpleNamespace(
            Keep=SimpleNamespace(ALL="all", LAST="last", NONE="none"),
            Request=lambda blocks, cached, tokens, keep, adapter=None: (cached, tokens, keep))

    def forward(self, reqs, cache, adapters=None):
        assert sum(len(t.values) for _, t, _ in reqs) <= self.rows
        self.calls.append(reqs)
        out = []
        for _, t, keep in reqs:
            if keep == "all":
                out += [v + 1 for v in t.values]
            elif keep == "last":
                out.append(t.values[-1] + 1)
        return _FakeTensor(out)


class _FakeHost:
    def __init__(self, a):
        self.a = a

    def to_hbm(self, device):
        return _FakeTensor(self.a.tolist())


def _runner(rows):
    from types import SimpleNamespace

    from furiosa_opt_vllm.runner import Runner

    eng = _FakeEngine(rows)
    r = Runner.__new__(Runner)
    r.engine, r.dec = SimpleNamespace(HostTensor=_FakeEngine.HostTensor), eng.dec
    r.model, r.device, r.cache, r.adapters, r.pooling_config, r.pooled, r.states = eng, None, None, None, None, [], {}
    r.uncollected = []
    return r, eng


def _sched(new=(), cached=(), counts=None):
    from types import SimpleNamespace

    cr = SimpleNamespace(req_ids=[c[0] for c in cached], new_block_ids=[None] * len(cached),
                         num_computed_tokens=[c[1] for c in cached], resumed_req_ids=set(), all_token_ids={})
    return SimpleNamespace(finished_req_ids=[], scheduled_new_reqs=list(new), scheduled_cached_reqs=cr,
                           num_scheduled_tokens=counts, scheduled_spec_decode_tokens={})


def test_runner_keeps_greedy_tokens_on_the_device_until_collected():
    """Async scheduling: step n+1 is issued before step n is collected; its input token is step n's
    device output, and the step is cut into calls of at most `rows` rows."""
    from types import SimpleNamespace

    runner, eng = _runner(rows=4)
    new = [SimpleNamespace(req_id=r, prompt_token_ids=p, num_computed_tokens=0, block_ids=([0, 1],))
           for r, p in (("a", [10, 11, 12]), ("b", [20, 21]))]
    first = runner.step(_sched(new=new, counts={"a": 3, "b": 2}), collect=False)
    assert len(eng.calls) == 2  # 5 rows over calls of 4
    second = runner.step(_sched(cached=[("a", 3), ("b", 2)], counts={"a": 1, "b": 1}), collect=False)
    # The decode rows read the first step's device outputs (13 and 22), never a host copy.
    assert [t.values for _, t, _ in eng.calls[-1]] == [[13], [22]]
    assert first.collect() == (["a", "b"], [[13], [22]])
    assert second.collect() == (["a", "b"], [[14], [23]])
    assert runner.states["a"].tokens == [10, 11, 12, 13, 14]
    third = runner.step(_sched(cached=[("a", 4), ("b", 3)], counts={"a": 1, "b": 1}))
    assert third == (["a", "b"], [[15], [24]])


def test_runner_of_a_rank_vllm_never_asks_collects_old_steps_itself():
    """Tensor-parallel ranks other than the driver are never asked for their tokens: each step
    collects every older step but the newest (whose token feeds it from the device)."""
    from types import SimpleNamespace

    runner, eng = _runner(rows=4)
    new = [SimpleNamespace(req_id="a", prompt_token_ids=[10, 11, 12], num_computed_tokens=0, block_ids=([0, 1],))]
    runner.step(_sched(new=new, counts={"a": 3}), collect=False)
    for i in range(4):
        runner.step(_sched(cached=[("a", 3 + i)], counts={"a": 1}), collect=False)
        assert len(runner.uncollected) <= 2
    # Every step's token came from the device; the tokens of all but the last two steps are known.
    assert runner.states["a"].tokens == [10, 11, 12, 13, 14, 15]
    assert [t.values for _, t, _ in eng.calls[-1]] == [[16]]


def test_block_tables_grow_and_resume():
    t = paging.BlockTable([3, 4])
    t.append([9])
    assert t.blocks == [3, 4, 9] and t.covers(48) and not t.covers(49)
    t.replace([1])
    assert t.blocks == [1]
    assert paging.first_group(([5, 6],)) == [5, 6]
    with pytest.raises(ValueError):
        paging.first_group(([1], [2]))


def test_request_state_schedules_and_samples():
    s = State([1, 2, 3, 4], 4, 0, paging.BlockTable([0]))
    assert s.scheduled(3) == [1, 2, 3] and not s.samples_after(3)
    s.computed = 3
    assert s.scheduled(1) == [4] and s.samples_after(1)
    with pytest.raises(ValueError):
        s.scheduled(2)


@pytest.mark.parametrize(("kwargs", "option"), [
    (dict(pipeline=2, tensor=1, speculative=None, lora=False, kv_cache_dtype="auto"), "pipeline_parallel_size"),
    (dict(pipeline=1, tensor=3, speculative=None, lora=False, kv_cache_dtype="auto"), "tensor_parallel_size"),
    (dict(pipeline=1, tensor=1, speculative="eagle", lora=False, kv_cache_dtype="auto"), "speculative_config"),
    (dict(pipeline=1, tensor=1, speculative=None, lora=True, kv_cache_dtype="auto", max_loras=3), "max_loras"),
    (dict(pipeline=1, tensor=1, speculative=None, lora=True, kv_cache_dtype="auto", max_lora_rank=64), "max_lora_rank"),
    (dict(pipeline=1, tensor=2, speculative=None, lora=True, kv_cache_dtype="auto"), "enable_lora"),
    (dict(pipeline=1, tensor=1, speculative=None, lora=False, kv_cache_dtype="fp8"), "kv_cache_dtype"),
])
def test_refusals_name_the_option(kwargs, option):
    with pytest.raises(admission.Refused) as e:
        admission.options(**kwargs)
    assert e.value.option == option
    admission.options(pipeline=1, tensor=8, speculative=None, lora=False, kv_cache_dtype="auto")


def test_sampling_refusals():
    admission.sampling(0.0, -1, 1.0, 1, None, None)
    with pytest.raises(admission.Refused):
        admission.sampling(0.7, -1, 1.0, 1, None, None)
    with pytest.raises(admission.Refused):
        admission.sampling(0.0, -1, 1.0, 1, 5, None)


def test_entry_point_names_the_platform():
    import furiosa_opt_vllm

    assert furiosa_opt_vllm.register() == "furiosa_opt_vllm.platform.B200Platform"


def test_replica_chips():
    from furiosa_opt_vllm import load

    # Consecutive GPUs of the replica whose tp_rank-th is this worker's.
    assert load.replica_chips(local_rank=5, tp_rank=1, tp=2) == [4, 5]
    assert load.replica_chips(local_rank=0, tp_rank=0, tp=1) == [0]
    # FURIOSA_VISIBLE_CHIPS lists every replica's chips in turn.
    assert load.replica_chips(0, 0, 2, dp_rank=1, visible="7,6,5,4") == [5, 4]
    with pytest.raises(ValueError, match="replica 2 of 2 chips needs 6"):
        load.replica_chips(0, 0, 2, dp_rank=2, visible="0,1,2,3")
    with pytest.raises(ValueError, match="cannot hold tensor-parallel rank 3"):
        load.replica_chips(local_rank=1, tp_rank=3, tp=4)


def test_lora_slots_follow_lru_and_pins():
    from types import SimpleNamespace

    from furiosa_opt_vllm import lora

    reads = []

    def read(req):
        reads.append(req.lora_int_id)
        return f"adapter{req.lora_int_id}"

    def req(i, inplace=False):
        return SimpleNamespace(lora_int_id=i, lora_name=f"l{i}", load_inplace=inplace)

    a = lora.Adapters(max_loras=2, max_cpu_loras=3, spec=None, read=read)
    assert a.activate({"r1": req(1), "r2": req(2)}) == {"r1": 0, "r2": 1}
    assert a.slots == ["adapter1", "adapter2"]
    # A third adapter takes the least recently used slot not in the step.
    assert a.activate({"r3": req(3)}) == {"r3": 0}
    assert a.ids() == {1, 2, 3} and reads == [1, 2, 3]
    # A fourth loaded adapter unloads the least recently used one (1).
    a.add(req(4))
    assert a.ids() == {2, 3, 4}
    # Pinned adapters keep their slots; a step needing more slots than unpinned ones is refused.
    a.pin(3)
    a.pin(4)
    with pytest.raises(RuntimeError, match="hold every slot"):
        a.activate({"r5": req(5)})
    assert a.remove(4) and not a.remove(4)
    # Loading in place reads the checkpoint again.
    a.add(req(3, inplace=True))
    assert reads[-1] == 3
    with pytest.raises(RuntimeError, match="above --max-loras"):
        a.activate({"x": req(7), "y": req(8), "z": req(9)})


def test_additional_config_section():
    from types import SimpleNamespace

    from furiosa_opt_vllm.additional import Section

    assert Section.parse(SimpleNamespace(additional_config={})).cuda_graphs is True
    assert Section.parse(SimpleNamespace(additional_config={"other": 1})).cuda_graphs is True
    assert Section.parse(SimpleNamespace(additional_config={"furiosa": {"cuda_graphs": False}})).cuda_graphs is False
    with pytest.raises(admission.Refused) as e:
        Section.parse(SimpleNamespace(additional_config={"furiosa": {"unknown": 1}}))
    assert e.value.option == "additional_config.furiosa.unknown"
    with pytest.raises(admission.Refused) as e:
        Section.parse(SimpleNamespace(additional_config={"furiosa": {"cuda_graphs": "yes"}}))
    assert e.value.option == "additional_config.furiosa.cuda_graphs"
    with pytest.raises(admission.Refused, match="beside the target"):
        Section.parse(SimpleNamespace(additional_config={"furiosa": {"draft_placement": {"chips": [1]}}}))
    with pytest.raises(admission.Refused) as e:
        Section.parse(SimpleNamespace(additional_config={"furiosa": {"draft_placement": {"chips": [1, 1]}}}))
    assert e.value.option.startswith("additional_config.furiosa.draft_placement")


def test_parameters_that_change_the_greedy_token_are_refused():
    from types import SimpleNamespace

    admission.unmodified(SimpleNamespace(repetition_penalty=1.0, min_tokens=0, logit_bias={}, bad_words=[],
                                         structured_outputs=None))
    for name, value in [("repetition_penalty", 1.1), ("frequency_penalty", 0.5), ("presence_penalty", -0.2),
                        ("min_tokens", 3), ("logit_bias", {5: 2.0}), ("allowed_token_ids", [1, 2]),
                        ("bad_words", ["x"]), ("structured_outputs", object()), ("extra_args", {"k": 1})]:
        with pytest.raises(admission.Refused) as e:
            admission.unmodified(SimpleNamespace(**{name: value}))
        assert e.value.option == name


def test_every_contract_names_an_option_of_this_vllm():
    """Each contract's path exists in vLLM's configuration classes (a renamed option would silently
    skip its check otherwise). The classes are read from vLLM's sources: importing vllm.config
    resolves vLLM's platform, which needs a GPU driver."""
    import ast
    import importlib.util
    from pathlib import Path

    spec = importlib.util.find_spec("vllm")
    if spec is None:
        pytest.skip("vLLM is not installed")
    fields: dict[str, set[str]] = {}
    for src in (Path(spec.origin).parent / "config").glob("*.py"):
        for node in ast.walk(ast.parse(src.read_text())):
            if isinstance(node, ast.ClassDef):
                names = {n.target.id for n in node.body if isinstance(n, ast.AnnAssign) and isinstance(n.target, ast.Name)}
                fields.setdefault(node.name, set()).update(names)
    classes = {"parallel_config": "ParallelConfig", "cache_config": "CacheConfig", "model_config": "ModelConfig",
               "load_config": "LoadConfig", "lora_config": "LoRAConfig", "scheduler_config": "SchedulerConfig",
               "offload_config": "OffloadConfig", "kv_transfer_config": "KVTransferConfig"}
    for c in admission.CONTRACTS:
        head, _, rest = c.path.partition(".")
        assert head in fields["VllmConfig"], c.path
        if rest:
            assert rest.split(".")[0] in fields[classes[head]], c.path


@pytest.mark.parametrize(("path", "bad", "option"), [
    ("parallel_config.nnodes", 2, "nnodes"),
    ("cache_config.cache_dtype", "fp8", "kv_cache_dtype"),
    ("model_config.dtype", "float16", "dtype"),
    ("model_config.quantization", "awq", "quantization"),
    ("load_config.load_format", "gguf", "load_format"),
    ("lora_config.fully_sharded_loras", True, "fully_sharded_loras"),
])
def test_contract_table_refuses_each_option(path, bad, option):
    from types import SimpleNamespace as ns

    def config():
        return ns(parallel_config=ns(pipeline_parallel_size=1, tensor_parallel_size=1, nnodes=1),
                  cache_config=ns(cache_dtype="auto"), model_config=ns(dtype="bfloat16", quantization=None),
                  load_config=ns(load_format="auto"), lora_config=ns(max_loras=1, max_lora_rank=8, fully_sharded_loras=False),
                  speculative_config=None, ec_transfer_config=None)

    admission.check(config())
    cfg = config()
    head, attr = path.split(".")
    setattr(getattr(cfg, head), attr, bad)
    with pytest.raises(admission.Refused) as e:
        admission.check(cfg)
    assert e.value.option == option


class _Transfer:
    def __init__(self, fn, fail=False):
        self.fn, self.fail, self.ran = fn, fail, False

    def done(self):
        return True

    def wait(self):
        if not self.ran:
            self.ran = True
            self.fn()
        if self.fail:
            raise RuntimeError("copy failed")


class _Buf:
    """A byte range of a bytearray standing for a device or pinned host buffer."""

    def __init__(self, data, off=0, n=None, fail=None):
        self.data, self.off, self.n, self.fail = data, off, len(data) - off if n is None else n, fail

    def slice(self, off, n):
        return _Buf(self.data, self.off + off, n, self.fail)

    def _to(self, other):
        def run():
            other.data[other.off : other.off + self.n] = self.data[self.off : self.off + self.n]
        return _Transfer(run, fail=self.fail is not None and self.fail())

    to_host = _to
    to_hbm = _to


def test_offload_pages_round_trip_and_poison_on_failure():
    """The KV offload handlers copy whole engine pages of every layer to host slots and back; a
    failed copy fails its job only once all its copies ended, and poisons later jobs."""
    from types import SimpleNamespace

    from furiosa_opt_vllm import offload

    page, layers, blocks = 8, 2, 4
    dev = [bytearray(bytes(range(l * 100, l * 100 + blocks * page))) for l in range(layers)]
    cache = SimpleNamespace(layers=[_Buf(d) for d in dev])
    host = bytearray(blocks * layers * page)
    pool = SimpleNamespace(page=page, layers=layers, poisoned=False,
                           slot=lambda b, l: _Buf(host, (b * layers + l) * page, page))
    store, load = offload.PageCopies(cache, pool, True), offload.PageCopies(cache, pool, False)
    ids = lambda *b: SimpleNamespace(block_ids=list(b))  # noqa: E731
    assert store.transfer_async(1, (ids(2, 0), ids(0, 3)))
    [r] = store.get_finished()
    assert (r.job_id, r.success, r.transfer_size) == (1, True, 2 * layers * page)
    want = [bytes(dev[l][2 * page : 3 * page]) for l in range(layers)]
    for l in range(layers):
        dev[l][2 * page : 3 * page] = bytes(page)  # the device block is reused
    assert load.transfer_async(2, (ids(0), ids(2)))
    load.wait({2})
    assert [bytes(dev[l][2 * page : 3 * page]) for l in range(layers)] == want
    assert [r.job_id for r in load.get_finished()] == [2]
    # A failing copy: the job fails after every copy ran, and the memory is poisoned afterwards.
    bad = SimpleNamespace(layers=[_Buf(d, fail=lambda: True) for d in dev])
    failing = offload.PageCopies(bad, pool, True)
    failing.transfer_async(3, (ids(1), ids(1)))
    with pytest.raises(RuntimeError, match="poisoned"):
        failing.wait({3})
    assert failing.get_finished()[0].success is False and pool.poisoned
    store.transfer_async(4, (ids(0), ids(0)))
    assert store.get_finished()[0].success is False


def test_encoder_caches_only_from_a_media_encoder_instance():
    from types import SimpleNamespace as ns

    def config(encoder_only, producer):
        return ns(parallel_config=ns(pipeline_parallel_size=1, tensor_parallel_size=1, nnodes=1),
                  cache_config=ns(cache_dtype="auto"),
                  model_config=ns(dtype="bfloat16", quantization=None,
                                  multimodal_config=ns(mm_encoder_only=encoder_only)),
                  load_config=ns(load_format="auto"), speculative_config=None,
                  ec_transfer_config=ns(is_ec_producer=producer))

    admission.check(config(True, True))
    for args in ((False, True), (True, False)):
        with pytest.raises(admission.Refused) as e:
            admission.check(config(*args))
        assert e.value.option == "ec_transfer_config"


class _Rows:
    def __init__(self, values):
        self.values = values
        self.shape = values.shape

    def to_host(self):
        return self

    def numpy(self):
        return self.values.float().numpy()


def test_media_step_embeds_each_item_once_and_frees_hashes():
    """An encoder-only step: scheduled images, video frames and audio embed through the engine's
    encoder with the processor's padding left out, each hash once, saved through the connector
    callback; freed hashes leave both caches."""
    from types import SimpleNamespace as ns

    import torch

    from furiosa_opt_vllm import media

    calls = []

    class Encoder:
        def vision(self, images):
            (im,) = images
            calls.append(("vision", im.pixels.shape[0], im.positions))
            return [_Rows(im.pixels * 2)]

        def audio(self, clips):
            (clip,) = clips
            calls.append(("audio", clip.frames.shape[0]))
            return [_Rows(clip.frames[:, :4])]

    class Host:
        @staticmethod
        def from_dlpack(t):
            return ns(to_hbm=lambda device: t)

    engine = ns(HostTensor=Host, vision_language=ns(Image=lambda pixels, positions: ns(pixels=pixels, positions=positions),
                                                   Audio=lambda frames: ns(frames=frames)))
    m = media.Media(engine, Encoder(), device=None)
    pix = torch.arange(12, dtype=torch.float32).reshape(3, 4)
    pos = torch.tensor([[0, 0], [1, 0], [-1, -1]])
    image = ns(identifier="img", modality="image", data={"pixel_values": pix, "pixel_position_ids": pos},
               mm_position=ns(get_num_embeds=lambda: 2))
    video = ns(identifier="vid", modality="video",
               data={"pixel_values_videos": torch.ones(2, 2, 4), "pixel_position_ids_videos": torch.zeros(2, 2, 2, dtype=torch.long)},
               mm_position=ns(get_num_embeds=lambda: 4))
    audio = ns(identifier="aud", modality="audio",
               data={"input_features_padded": torch.ones(5, 8), "input_features_mask": torch.tensor([1, 1, 1, 0, 0])},
               mm_position=ns(get_num_embeds=lambda: 3))
    so = ns(finished_req_ids=set(), free_encoder_mm_hashes=[],
            scheduled_new_reqs=[ns(req_id="a", mm_features=[image, video]), ns(req_id="b", mm_features=[audio, image])],
            scheduled_encoder_inputs={"a": [0, 1], "b": [0, 1]})
    saved = []
    done = m.step(so, save=lambda cache, h: saved.append((h, cache[h].dtype)))
    assert done == ["img", "vid", "aud"]  # the second request's image hash was embedded already
    assert saved == [("img", torch.bfloat16), ("vid", torch.bfloat16), ("aud", torch.bfloat16)]
    assert calls[0] == ("vision", 2, [[0, 0], [1, 0]]) and calls[1][:2] == ("vision", 4) and calls[2] == ("audio", 3)
    assert torch.equal(m.host["img"].float(), pix[:2] * 2)
    so2 = ns(finished_req_ids={"a"}, free_encoder_mm_hashes=["img", "vid"], scheduled_new_reqs=[],
             scheduled_encoder_inputs={})
    assert m.step(so2) == []
    assert set(m.host) == {"aud"} and set(m.rows) == {"aud"} and set(m.features) == {"b"}
    bad = ns(identifier="x", modality="image", data={"pixel_values": pix, "pixel_position_ids": pos},
             mm_position=ns(get_num_embeds=lambda: 3))
    with pytest.raises(ValueError, match="placeholders"):
        m.embed(bad)


def test_config_overrides_apply_to_the_checkpoint_config(tmp_path):
    """vLLM's `hf_overrides` (a mapping) replace config.json keys as transformers' update does; a
    nested sub-config is updated key by key; a function of the config is refused."""
    import json

    from furiosa_opt_vllm import load

    (tmp_path / "config.json").write_text(json.dumps({
        "architectures": ["Qwen3ForCausalLM"], "max_position_embeddings": 4096, "rope_theta": 1e6,
        "rope_scaling": {"rope_type": "linear", "factor": 2.0}, "text_config": {"model_type": "x", "a": 1, "b": 2}}))
    assert load.overridden(str(tmp_path), None) is None
    assert load.overridden(str(tmp_path), {}) is None
    got = load.overridden(str(tmp_path), {"rope_scaling": {"rope_type": "yarn", "factor": 4.0,
                                                            "original_max_position_embeddings": 4096},
                                          "max_position_embeddings": 16384, "text_config": {"b": 3}})
    assert got["rope_scaling"] == {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 4096}
    assert got["max_position_embeddings"] == 16384 and got["rope_theta"] == 1e6
    assert got["text_config"] == {"model_type": "x", "a": 1, "b": 3}
    with pytest.raises(admission.Refused) as e:
        load.overridden(str(tmp_path), lambda c: c)
    assert e.value.option == "hf_overrides"


def test_overridden_config_reaches_the_engine_load(tmp_path):
    """The overridden config is what the registry reads: YaRN scaling selects, a refused scaling is
    refused by the registry with its key."""
    import json

    import furiosa_opt_engine as engine
    from furiosa_opt_models_b200.models import configs, synthetic
    from furiosa_opt_vllm import load

    (tmp_path / "config.json").write_text(json.dumps(synthetic.hf_config(configs.get("qwen3-1.7b"))))
    ok = load.overridden(str(tmp_path), {"rope_scaling": {"rope_type": "yarn", "factor": 4.0,
                                                           "original_max_position_embeddings": 40960}})
    assert engine.LoadOptions().select(load.checkpoint(str(tmp_path), ok))["class"] == "qwen3.ForCausalLM"
    bad = load.overridden(str(tmp_path), {"rope_scaling": {"rope_type": "longrope", "factor": 4.0}})
    with pytest.raises(NotImplementedError, match="rope_scaling"):
        engine.LoadOptions().select(load.checkpoint(str(tmp_path), bad))


def test_batch_invariant_vllm_loads_batch_invariant(monkeypatch):
    import furiosa_opt_engine as engine
    from furiosa_opt_vllm import load

    calls = []

    class Options:
        def __init__(self):
            self.chain = []

        def __getattr__(self, name):
            def step(*args):
                self.chain.append((name, args))
                return self
            return step

        def load(self, ck, device):
            calls.append(self.chain)
            return "decoder"

    monkeypatch.setattr(engine, "LoadOptions", Options)
    monkeypatch.setenv("VLLM_BATCH_INVARIANT", "1")
    assert load.batch_invariant()
    load.load_from("ck", "dev", 2)
    monkeypatch.setenv("VLLM_BATCH_INVARIANT", "0")
    load.load_from("ck", "dev", 1)
    load.load_from("ck", "dev", 1, invariant=True)
    assert [[n for n, _ in c] for c in calls] == [["chips", "batch_invariant"], [], ["batch_invariant"]]


def test_overrides_contract():
    from types import SimpleNamespace as ns

    cfg = ns(parallel_config=ns(pipeline_parallel_size=1, tensor_parallel_size=1, nnodes=1),
             cache_config=ns(cache_dtype="auto"),
             model_config=ns(dtype="bfloat16", quantization=None, hf_overrides={"max_position_embeddings": 8192}),
             load_config=ns(load_format="auto"), speculative_config=None, ec_transfer_config=None)
    admission.check(cfg)
    cfg.model_config.hf_overrides = lambda c: c
    with pytest.raises(admission.Refused) as e:
        admission.check(cfg)
    assert e.value.option == "hf_overrides"


def test_thinking_budget_forces_the_end_marker():
    from furiosa_opt_vllm import thinking

    start, end = [100], [101, 102]
    b = thinking.Budget(3, start, end)
    b.reset([5, 6])
    out = [b.choose(t) for t in [100, 7, 8, 9, 10, 11, 12, 13]]
    # Three thinking tokens after the start marker, then the two end tokens, then the model again.
    assert out == [100, 7, 8, 9, 101, 102, 12, 13]
    b = thinking.Budget(5, start, end)
    b.reset([5])
    assert [b.choose(t) for t in [100, 7, 101, 102, 8, 9, 10, 11, 12, 13]] == [100, 7, 101, 102, 8, 9, 10, 11, 12, 13]
    b = thinking.Budget(0, start, end)
    b.reset([5, 100], prompt=2)  # the prompt opens the section: no token of thought is allowed
    assert [b.choose(t) for t in [7, 8, 9]] == [101, 102, 9]
    b = thinking.Budget(2, [], [101])  # no start marker: thinking from the first token
    b.reset([1, 2, 3], prompt=3)
    assert [b.choose(t) for t in [7, 8, 9]] == [7, 8, 101]
    with pytest.raises(ValueError):
        thinking.Budget(2, start, [])


def test_runner_applies_thinking_budgets_and_feeds_forced_tokens():
    """The fake engine's token is its input + 1; a budget of 2 after the start marker 13 forces the
    end marker 50, which the next step feeds from the host."""
    from types import SimpleNamespace

    runner, eng = _runner(rows=8)
    runner.reasoning = ([13], [50])
    new = [SimpleNamespace(req_id="a", prompt_token_ids=[10, 11, 12], num_computed_tokens=0, block_ids=([0, 1],),
                           sampling_params=SimpleNamespace(thinking_token_budget=2))]
    got = [runner.step(_sched(new=new, counts={"a": 3}))[1][0]]
    for i in range(5):
        got.append(runner.step(_sched(cached=[("a", 3 + i)], counts={"a": 1}))[1][0])
    # 13 opens thinking; 14 and 15 spend the budget; 50 is forced; 51, 52 follow it.
    assert [g[0] for g in got] == [13, 14, 15, 50, 51, 52]
    assert [t.values for _, t, _ in eng.calls[4]] == [[50]]
    assert runner.states["a"].tokens == [10, 11, 12, 13, 14, 15, 50, 51, 52]
    assert runner.reads_each_step(_sched(cached=[("a", 9)], counts={"a": 1}))


def test_a_forced_token_drops_the_accepted_drafts_after_it():
    from furiosa_opt_vllm import thinking
    from furiosa_opt_vllm.request import State

    b = thinking.Budget(1, [13], [50])
    b.reset([13], prompt=1)
    st = State([13], 1, 1, None, budget=b)
    # Speculative step: the engine's tokens 20, 21, 22 were accepted; the budget forces 50 after 20.
    assert thinking.apply(st.budget, [20, 21, 22]) == [20, 50]


def test_budgets_need_reasoning_markers():
    from types import SimpleNamespace

    runner, _ = _runner(rows=8)
    runner.reasoning = None
    new = [SimpleNamespace(req_id="a", prompt_token_ids=[10], num_computed_tokens=0, block_ids=([0],),
                           sampling_params=SimpleNamespace(thinking_token_budget=2))]
    with pytest.raises(ValueError, match="reasoning-parser"):
        runner.step(_sched(new=new, counts={"a": 1}))
