"""The tensor-parallel all-reduce's schedule on the host, against the contract's result (a
rank-ordered FP32 sum, one rounding, then the norm) over consecutive calls: slots, buffers and marks
of the CUDA collective run rank by rank in Python (furiosa_opt_models_b200.parallel.emulate), and the
same schedule on concurrently running rank threads in C++ (csrc/engine/comm_emulate.cc)."""

import numpy as np
import pytest

from furiosa_opt_models_b200.parallel import emulate


def _call_inputs(rng, world, rows, cols):
    partials = [rng.standard_normal((rows, cols)).astype(np.float32) for _ in range(world)]
    partials[0][0, 0] = np.float32(-0.0)  # a -0.0 sum travels as +0.0
    residual = emulate.bf16(rng.standard_normal((rows, cols)).astype(np.float32))
    weight = emulate.bf16(rng.standard_normal(cols).astype(np.float32))
    return partials, residual, weight


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("rows", [1, 7, 64, 300])
@pytest.mark.parametrize("one_shot_bytes", [4 << 20, 0])
def test_schedule_matches_the_rank_ordered_sum(world, rows, one_shot_bytes):
    cols = 64
    rng = np.random.default_rng(world * 1000 + rows)
    hs = emulate.heaps(world, 300, cols)
    residuals = None
    for call in range(3):  # both receive buffers, then the first again
        partials, residual, weight = _call_inputs(rng, world, rows, cols)
        residuals = [residual.copy() for _ in range(world)]
        hidden = emulate.add_norm(hs, partials, residuals, weight, 1e-6, one_shot_bytes=one_shot_bytes,
                                  gather_residual=True)
        want_x, want_h = emulate.rank_ordered(partials, residual, weight, 1e-6)
        for q in range(world):
            assert np.array_equal(hidden[q], want_h), (call, q)
            assert np.array_equal(residuals[q], want_x), (call, q)
    # Every slot is marked unwritten again after its reduction.
    for h in hs:
        assert bool(emulate.is_unwritten(h.recv).all())


def test_reduce_scatter_keeps_each_residual_row_on_its_owner():
    world, rows, cols = 4, 10, 32
    rng = np.random.default_rng(3)
    hs = emulate.heaps(world, rows, cols)
    partials, residual, weight = _call_inputs(rng, world, rows, cols)
    residuals = [residual.copy() for _ in range(world)]
    emulate.add_norm(hs, partials, residuals, weight, 1e-6, one_shot_bytes=0, gather_residual=False)
    want_x, _ = emulate.rank_ordered(partials, residual, weight, 1e-6)
    owner = (rows + world - 1) // world
    for q in range(world):
        for r in range(rows):
            expect = want_x[r] if r // owner == q else residual[r]
            assert np.array_equal(residuals[q][r], expect)


def test_rows_past_the_slots_take_reduce_scatter():
    # One-shot needs every row in one slot: a call of more rows than a slot holds reduce-scatters.
    assert emulate.two_shot(rows=80, cols=64, world=4, slot_rows=75)
    assert not emulate.two_shot(rows=75, cols=64, world=4, slot_rows=75)
    assert emulate.two_shot(rows=8, cols=2048, world=8, slot_rows=64, one_shot_bytes=0)


@pytest.mark.parametrize("rows,cols,kbn,splits", [(64, 256, 64, 4), (3, 384, 16, 8), (100, 128, 128, 2)])
def test_gemm_split_layout_adds_up_in_split_order(rows, cols, kbn, splits):
    """A decode GEMM's K splits in the GemmSplits layout: every (split, token, feature) has its own
    slot, and the reducer's sum in split order equals the sum of the per-split partials."""
    rng = np.random.default_rng(rows + cols)
    tiles_p = (cols + 127) // 128
    tiles_q = (rows + kbn - 1) // kbn
    per = [rng.standard_normal((rows, cols)).astype(np.float32) for _ in range(splits)]
    ws = np.full(tiles_p * tiles_q * splits * 128 * kbn, np.nan, dtype=np.float32)
    seen = set()
    for s in range(splits):
        for t in range(rows):
            for f in range(cols):
                i = emulate.splits_at(s, t, f, splits, kbn, tiles_p)
                assert i not in seen
                seen.add(i)
                ws[i] = per[s][t, f]
    want = np.zeros((rows, cols), dtype=np.float32)
    for p in per:
        want = (want + p).astype(np.float32)
    assert np.array_equal(emulate.split_sum(ws, rows, cols, splits, kbn, tiles_p), want)


# ---- The same schedule on host threads (csrc/engine/comm_emulate.cc): ranks run concurrently ----

def _bits(x: np.ndarray) -> np.ndarray:
    return (emulate.bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def _from_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def _threaded_call(rng, world, rows, cols, gather=False):
    partials = [rng.standard_normal((rows, cols)).astype(np.float32) for _ in range(world)]
    partials[world - 1][0, :8] = np.float32(-0.0)  # -0.0 travels as +0.0
    residual = emulate.bf16(rng.standard_normal((rows, cols)).astype(np.float32))
    weight = emulate.bf16(rng.standard_normal(cols).astype(np.float32))
    call = {"rows": rows, "cols": cols, "partials": partials, "residual": _bits(residual), "weight": _bits(weight),
            "eps": 1e-6, "gather_residual": gather}
    return call, emulate.rank_ordered(partials, residual, weight, 1e-6)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize(("one_shot_bytes", "inline_rows"), [(4 << 20, 148), (4 << 20, 0), (0, 148), (0, 0)],
                         ids=["one-shot-inline", "one-shot-scatter", "two-shot-inline", "two-shot-scatter"])
def test_threaded_ranks_match_the_rank_ordered_sum(world, one_shot_bytes, inline_rows):
    """Six consecutive calls of different row counts (both receive buffers, twice) on concurrently
    running rank threads, with random yields: every rank's residual rows are the rank-ordered FP32
    sum plus the residual, rounded once (bitwise), and the normed rows agree to a BF16 step."""
    from furiosa_opt_engine import _native

    rng = np.random.default_rng(world * 17 + one_shot_bytes % 7 + inline_rows)
    cols = 64
    calls, wants = [], []
    for rows in (1, 9, 40, 3, 40, 17):
        c, w = _threaded_call(rng, world, rows, cols)
        calls.append(c)
        wants.append(w)
    out = _native._tp_emulate(world, calls, slot_rows=40, one_shot_bytes=one_shot_bytes, inline_rows=inline_rows,
                              jitter_seed=7)
    assert out["timeouts"] == [0] * world
    assert all(out["two_shot"]) == (one_shot_bytes == 0)
    for n, (call_out, (want_x, want_h)) in enumerate(zip(out["calls"], wants)):
        rows = calls[n]["rows"]
        owner = (rows + world - 1) // world
        for q, (hidden, residual) in enumerate(call_out):
            got_x = _from_bits(residual)
            mine = [r for r in range(rows) if one_shot_bytes or r // owner == q]
            assert np.array_equal(got_x[mine], want_x[mine]), (n, q)
            np.testing.assert_allclose(_from_bits(hidden), want_h, rtol=2 ** -7, atol=1e-6)


def test_threaded_two_shot_gathers_residual_rows_when_asked():
    from furiosa_opt_engine import _native

    rng = np.random.default_rng(5)
    world, rows, cols = 4, 10, 32
    call, (want_x, _) = _threaded_call(rng, world, rows, cols, gather=True)
    out = _native._tp_emulate(world, [call], slot_rows=16, one_shot_bytes=0, jitter_seed=3)
    for _, residual in out["calls"][0]:
        assert np.array_equal(_from_bits(residual), want_x)


def test_a_rank_that_never_pushes_ends_its_peers_waits_with_timeouts():
    """A rank that scatters nothing: every rank's polls for its slot run out after the limit and are
    counted (the kernels record a peer-timeout status and return); the call still ends."""
    from furiosa_opt_engine import _native

    rng = np.random.default_rng(9)
    call, _ = _threaded_call(rng, 2, 4, 16)
    out = _native._tp_emulate(2, [call], slot_rows=4, wait_limit_s=0.05, drop_rank=1)
    assert all(t > 0 for t in out["timeouts"])


def test_emulation_refuses_calls_that_do_not_fit_the_slots():
    from furiosa_opt_engine import _native

    rng = np.random.default_rng(1)
    call, _ = _threaded_call(rng, 2, 8, 16)  # 8 rows past 4-row slots go two-shot: 4 rows a rank
    assert _native._tp_emulate(2, [call], slot_rows=4, one_shot_bytes=1 << 30)["two_shot"] == [True]
    call, _ = _threaded_call(rng, 2, 9, 16)  # 5 rows a rank do not fit
    with pytest.raises(Exception, match="receive slots"):
        _native._tp_emulate(2, [call], slot_rows=4, one_shot_bytes=1 << 30)
