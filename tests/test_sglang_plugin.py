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
