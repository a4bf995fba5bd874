"""The batch planner's rules, each refusal by kind and message (the reference planner's own:
crates/furiosa-opt-engine/src/decoder/batch/mod.rs), and its layout of call rows."""

import pytest

from furiosa_opt_engine import _native

POOL = [(16, 64)]
GROUP = [(0, 0, 1, "paged", 0, None)]


def plan(requests, window=64, rows=8, blocks=64, pools=POOL, groups=GROUP, cache_pools=None,
         cache_groups=None, adapters_limit=0, adapters_given=0, filled=(), group=1):
    return _native._plan(requests, window, rows, adapters_limit, pools, groups,
                         cache_pools if cache_pools is not None else pools,
                         cache_groups if cache_groups is not None else groups, blocks, adapters_given,
                         list(filled), group)


def req(blocks, cached, length, **kw):
    return dict(rows=[list(blocks)], cached=cached, length=length, **kw)


def test_lays_out_one_row_requests_first():
    assert _native._layout([3, 1, 2, 1]) == [(2, 5), (0, 1), (5, 7), (1, 2)]


def test_keeps_selected_rows_in_request_order():
    p = plan([req([7], 5, 1), req([2], 0, 2, keep="none"), req([5], 0, 2, keep="all"),
              req([6], 0, 3, keep=(1, 3))])
    assert p["kept"] == [0, 3, 4, 6, 7]


def test_accepts_any_block_past_the_used_ones():
    plan([req([7, 5, 99], 3, 2)], pools=[(4, 64)], blocks=8)


def test_positions_and_slots():
    p = plan([req([3, 9], 14, 4)])
    assert p["positions"] == [14, 15, 16, 17]
    assert p["slots"] == [3 * 16 + 14, 3 * 16 + 15, 9 * 16 + 0, 9 * 16 + 1]
    assert p["segments"] == [0, 4, 14, 0, 2]


@pytest.mark.parametrize(
    "requests,kw,message",
    [
        ([], {}, "call has no requests"),
        ([req([7], 0, 1)], {"cache_pools": [(4, 64)]}, "cache was allocated for another model"),
        ([dict(rows=[[7], [8]], cached=0, length=1)], {}, "request holds a block list for each cache group"),
        ([req([7], 0, 0)], {}, "request has no tokens"),
        ([req([7], 2, 3)], {"window": 4}, "request extends past the context window"),
        ([req(list(range(17)), 1 << 24, 1)], {"window": (1 << 24) + 1, "pools": [(1 << 20, 64)]},
         "position is not below 2\\^24"),
        ([req([7], 15, 2)], {}, "request has fewer blocks than its positions need"),
        ([req([64], 0, 1)], {}, "block ID is outside the cache"),
        ([req([7], 0, 1, keep=(0, 2))], {}, "kept rows lie outside the appended rows"),
        ([req([7], 0, 1, keep=(1, 0))], {}, "kept rows lie outside the appended rows"),
        ([req([7], 0, 9)], {}, "call has more rows than compiled"),
        ([req([7], 0, 1), req([7], 0, 1)], {}, "two appended positions share a cache slot"),
    ],
)
def test_refuses_invalid_requests(requests, kw, message):
    with pytest.raises(ValueError, match=f"^{message}$"):
        plan(requests, **kw)


def test_empty_kept_range_is_accepted():
    assert plan([req([7], 0, 1, keep=(1, 1))])["kept"] == []


@pytest.mark.parametrize(
    "flag,message",
    [
        ({"adapter": 0}, "adapters are not served"),
        ({"positions": True}, "explicit positions are not served"),
        ({"mask": True}, "visibility masks are not served"),
        ({"overrides": True}, "row overrides are not served"),
    ],
)
def test_refuses_unserved_requests(flag, message):
    with pytest.raises(NotImplementedError, match=f"^{message}$"):
        plan([req([7], 0, 1, **flag)])


@pytest.mark.parametrize("groups", [[(0, 0, 1, "state", 0, None)], [(0, 0, 1, "cross", 4, None)], []])
def test_refuses_groups_other_than_paged(groups):
    with pytest.raises(NotImplementedError, match="^a call plans paged cache groups$"):
        plan([req([7], 0, 1)], groups=groups)


def test_refuses_unheld_adapters():
    with pytest.raises(ValueError, match="^call holds more adapters than compiled$"):
        plan([req([7], 0, 1, adapter=0)], adapters_limit=2, adapters_given=3, filled=[True] * 3)
    with pytest.raises(ValueError, match="^request names a slot that holds no adapter$"):
        plan([req([7], 0, 1, adapter=1)], adapters_limit=2, adapters_given=2, filled=[True, False])
    with pytest.raises(ValueError, match="^request names a slot that holds no adapter$"):
        plan([req([7], 0, 1, adapter=2)], adapters_limit=2, adapters_given=2, filled=[True, True])


def test_prefill_work_tiles():
    # Query tiles hold 128 (token, head) rows: 33 rows x 2 heads fit one tile, 65 x 2 need two.
    p = plan([req([1, 2, 3], 0, 33), req([9], 4, 1)], rows=128, group=2)
    assert p["decode"] == 1 and p["prefill"] == 1
    assert p["work"] == [1, 0]
    p = plan([req([1, 2, 3, 4, 5], 0, 65), req([9], 4, 1)], rows=128, group=2, window=128)
    assert p["work"] == [1, 0, 1, 1]
