"""A host model of the tensor-parallel all-reduce's data movement, the oracle of its schedule.

The CUDA collective (csrc/kernels/comm.cu, csrc/engine/comm.cc) moves FP32 partials between ranks
through receive slots in every rank's symmetric heap; this module runs the same schedule on numpy
arrays, rank by rank, so its layout and ordering rules can be checked on a CPU:

- Receive region of rank q: [2 buffers][world source slots][slot rows][cols] FP32, every value
  -0.0 ("not written") until a partial lands; the buffer is the low bit of a per-rank call
  sequence, so two consecutive calls never share one.
- One-shot (at most `one_shot_bytes` of pushed partials, and rows <= slot rows): rank p stores its
  row r into slot p, slot row r, of every rank. Reduce-scatter: row r goes to the rank
  q = r // ceil(rows / world) that owns it, at slot row r - q * ceil(rows / world).
- A pushed -0.0 is sent as +0.0, so the mark stays unambiguous; the reducer waits until none of its
  values is -0.0, adds the ranks' values in rank order in FP32 starting from +0.0, writes -0.0
  back, adds the BF16 residual (one rounding) and normalises; under reduce-scatter the owner
  stores the normed rows into every rank.
- A decode GEMM may leave its K splits instead of one partial (`splits_at`, the GemmSplits
  layout); the reducer adds them in split order before pushing.

The reference's contract (a deterministic rank-ordered FP32 sum rounded once):
crates/furiosa-opt-models/src/ops/collective/mod.rs:22-141.
"""

from __future__ import annotations

import dataclasses

import numpy as np

UNWRITTEN = np.float32(-0.0)


def bf16(x: np.ndarray) -> np.ndarray:
    """Rounds FP32 values to BF16 (round to nearest even), returned as FP32."""
    x = np.asarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    return rounded.astype(np.uint32).view(np.float32)


def is_unwritten(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).view(np.uint32) == np.uint32(0x80000000)


@dataclasses.dataclass
class Heap:
    """One rank's part of the symmetric heap that the collective uses."""

    recv: np.ndarray  # [2, world, slot_rows, cols] FP32
    seq: int = 0


def heaps(world: int, rows: int, cols: int) -> list[Heap]:
    slot_rows = (rows + world - 1) // world
    return [Heap(np.full((2, world, slot_rows, cols), UNWRITTEN, dtype=np.float32)) for _ in range(world)]


def two_shot(rows: int, cols: int, world: int, slot_rows: int, one_shot_bytes: int = 4 << 20) -> bool:
    return rows * cols * 4 * (world - 1) > one_shot_bytes or rows > slot_rows


def splits_at(s: int, t: int, f: int, splits: int, kbn: int, tiles_p: int) -> int:
    """Index of split s, token t, feature f in a GEMM's external split partials (GemmSplits::at)."""
    return ((f // 128 + (t // kbn) * tiles_p) * splits + s) * 128 * kbn + (t % kbn) * 128 + f % 128


def split_sum(ws: np.ndarray, rows: int, cols: int, splits: int, kbn: int, tiles_p: int) -> np.ndarray:
    """The partial [rows, cols] a GEMM's K splits add up to, in split order from +0.0."""
    out = np.zeros((rows, cols), dtype=np.float32)
    for s in range(splits):
        for t in range(rows):
            idx = [splits_at(s, t, f, splits, kbn, tiles_p) for f in range(cols)]
            out[t] = out[t] + ws[idx]
    return out


def add_norm(hs: list[Heap], partials: list[np.ndarray], residuals: list[np.ndarray], weight: np.ndarray,
             eps: float, one_shot_bytes: int = 4 << 20, gather_residual: bool = False):
    """Runs one call of the collective over every rank: scatter, then each rank's reduction.

    `partials[p]` is rank p's FP32 partial [rows, cols]; `residuals[p]` its BF16 residual stream
    (FP32 holding BF16 values), updated in place where the rank holds the row. Returns every rank's
    normed rows [rows, cols] (BF16 values)."""
    world = len(hs)
    rows, cols = partials[0].shape
    slot_rows = hs[0].recv.shape[2]
    two = two_shot(rows, cols, world, slot_rows, one_shot_bytes)
    owner_rows = (rows + world - 1) // world if two else 0
    # Scatter: every rank stores its rows into the reducing ranks' slots.
    for p in range(world):
        parity = hs[p].seq & 1
        part = np.where(is_unwritten(partials[p]), np.float32(0.0), partials[p]).astype(np.float32)
        for r in range(rows):
            dests = [r // owner_rows] if two else range(world)
            for q in dests:
                slot_row = r - q * owner_rows if two else r
                if not bool(is_unwritten(hs[q].recv[parity, p, slot_row]).all()):
                    raise AssertionError(f"rank {p} overwrote slot row {slot_row} of rank {q} before it was read")
                hs[q].recv[parity, p, slot_row] = part[r]
    # Reduction: each rank adds its slot rows in rank order, then residual and norm.
    hidden = [np.zeros((rows, cols), dtype=np.float32) for _ in range(world)]
    w = weight.astype(np.float32)
    for q in range(world):
        parity = hs[q].seq & 1
        mine = range(q * owner_rows, min(rows, (q + 1) * owner_rows)) if two else range(rows)
        for r in mine:
            slot_row = r - q * owner_rows if two else r
            acc = np.zeros(cols, dtype=np.float32)
            for p in range(world):
                got = hs[q].recv[parity, p, slot_row]
                if bool(is_unwritten(got).any()):
                    raise AssertionError(f"rank {q} reduced slot row {slot_row} before rank {p}'s row landed")
                acc = (acc + got).astype(np.float32)
                hs[q].recv[parity, p, slot_row] = UNWRITTEN
            x = bf16(acc + residuals[q][r])
            inv = np.float32(1.0) / np.sqrt(np.float32(np.mean(x.astype(np.float64) ** 2)) + np.float32(eps))
            h = bf16(x * np.float32(inv) * w)
            owners = range(world) if two else [q]
            for o in owners:
                hidden[o][r] = h
                if not two or gather_residual or o == q:
                    residuals[o][r] = x
    for h in hs:
        h.seq += 1
    return hidden


def rank_ordered(partials: list[np.ndarray], residual: np.ndarray, weight: np.ndarray, eps: float):
    """The contract's result computed directly: FP32 sum in rank order, one rounding, the norm."""
    acc = np.zeros_like(partials[0], dtype=np.float32)
    for p in partials:
        acc = (acc + np.where(is_unwritten(p), np.float32(0.0), p)).astype(np.float32)
    x = bf16(acc + residual)
    out = np.zeros_like(x)
    for r in range(x.shape[0]):
        inv = np.float32(1.0) / np.sqrt(np.float32(np.mean(x[r].astype(np.float64) ** 2)) + np.float32(eps))
        out[r] = bf16(x[r] * np.float32(inv) * weight.astype(np.float32))
    return x, out
