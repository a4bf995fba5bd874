"""The plugin's host contracts without a GPU: batch framing and planning, block tables, request
state, refusals."""

import pickle

import pytest

from furiosa_opt_vllm import admission, batch, paging
from furiosa_opt_vllm.request import State


def test_call_groups_chunks_and_keeps_last_rows():
    rows = (batch.Row("a", 5, False), batch.Row("a", 6, True), batch.Row("b", 0, False))
    call = batch.Call[str].plan(rows, every=False)
    assert call.requests == (batch.Request("a", 5, (0, 1), True), batch.Request("b", 0, (2,), False))
    assert call.kept == (1,)
    assert batch.Call[int].plan((batch.Row(0, 4, False), batch.Row(1, 0, True)), every=True).kept == (0, 1)


def test_batch_copies_tokens_and_derives_history():
    tokens = [1, 2, 3]
    parsed = batch.Batch.parse(tokens, [2, 1], [7, 1])
    tokens[0] = 9
    assert parsed.tokens == ((1, 2), (3,))
    assert parsed.cached == (5, 0)


@pytest.mark.parametrize(("tokens", "lengths", "totals"), [([1], [2], [2]), ([1, 1], [0, 2], [1, 2]), ([1], [1], [0])])
def test_batch_refuses_bad_framing(tokens, lengths, totals):
    with pytest.raises(batch.Framing) as e:
        batch.Batch.parse(tokens, lengths, totals)
    restored = pickle.loads(pickle.dumps(e.value))
    assert (restored.tokens, restored.scheduled) == (e.value.tokens, e.value.scheduled)


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
    with pytest.raises(admission.Refused, match="draft models are not served"):
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
