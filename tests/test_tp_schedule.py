"""The tensor-parallel all-reduce's schedule on the host (furiosa_opt_models_b200.parallel.emulate):
slots, buffers and marks of the CUDA collective, run rank by rank against the contract's result (a
rank-ordered FP32 sum, one rounding, then the norm), over consecutive calls."""

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
