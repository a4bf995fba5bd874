"""Torch-facing wrappers of the raw kernel launchers."""

from __future__ import annotations

import torch

from .native import native, scratch

EPI_BF16, EPI_F32, EPI_SWIGLU = 0, 1, 2
MODE_AUTO, MODE_ROWS, MODE_SWAP = 0, 1, 2


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.data_ptr()


def _rowmajor(t: torch.Tensor, name: str) -> None:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D tensor with unit column stride")


def gemm(
    a: torch.Tensor,
    w: torch.Tensor,
    epilogue: int = EPI_BF16,
    residual: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    mode: int = MODE_AUTO,
    splits: int = 0,
    trace: torch.Tensor | None = None,
) -> torch.Tensor:
    """``epilogue(a @ w.T)`` on the tcgen05 GEMM: a [M, K] BF16, w [N, K] BF16.

    EPI_BF16 returns BF16 [M, N] (plus ``residual`` before the one rounding), EPI_F32 FP32 [M, N],
    EPI_SWIGLU BF16 [M, N/2] for gate/up weights interleaved in 128-row blocks.
    """
    _rowmajor(a, "a")
    _rowmajor(w, "w")
    if a.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("gemm takes BF16 operands")
    M, K = a.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError("inner dimensions differ")
    cols = N // 2 if epilogue == EPI_SWIGLU else N
    if out is None:
        dtype = torch.float32 if epilogue == EPI_F32 else torch.bfloat16
        out = torch.empty(M, cols, dtype=dtype, device=a.device)
    if residual is not None:
        _rowmajor(residual, "residual")
    s = scratch(a.device)
    native().ops.gemm(
        a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), M, N, K,
        out.data_ptr(), out.stride(0), _ptr(residual), 0 if residual is None else residual.stride(0),
        epilogue, mode, splits, s.workspace.data_ptr(), s.workspace.numel() * 4,
        s.counters.data_ptr(), s.counters.numel(), s.status.data_ptr(), _stream(),
        0 if trace is None else trace.data_ptr(),
    )
    return out


def rmsnorm(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    residual: torch.Tensor | None = None,
    residual_out: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``RMSNorm(x + residual) * weight``; the rounded sum goes to ``residual_out`` when given."""
    _rowmajor(x, "x")
    rows, cols = x.shape
    out = torch.empty_like(x) if out is None else out
    native().ops.rmsnorm(
        x.data_ptr(), x.stride(0), _ptr(residual), 0 if residual is None else residual.stride(0),
        weight.data_ptr(), out.data_ptr(), out.stride(0), _ptr(residual_out),
        0 if residual_out is None else residual_out.stride(0), rows, cols, float(eps), _stream(),
    )
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, row_begin: int = 0, row_end: int | None = None) -> torch.Tensor:
    rows = ids.numel()
    row_end = table.shape[0] + row_begin if row_end is None else row_end
    out = torch.empty(rows, table.shape[1], dtype=table.dtype, device=table.device)
    native().ops.embedding(ids.data_ptr(), table.data_ptr(), table.stride(0), row_begin, row_end,
                           out.data_ptr(), out.stride(0), rows, table.shape[1], _stream())
    return out


def argmax(logits: torch.Tensor, valid: int | None = None, base: int = 0):
    rows, cols = logits.shape
    idx = torch.empty(rows, dtype=torch.int32, device=logits.device)
    val = torch.empty(rows, dtype=torch.float32, device=logits.device)
    native().ops.argmax(logits.data_ptr(), logits.stride(0), rows, cols,
                        cols if valid is None else valid, base, idx.data_ptr(), val.data_ptr(),
                        _stream())
    return idx, val


def qk_norm_rope_cache(qkv, q_heads, kv_heads, head_dim, q_norm, k_norm, eps, positions, inv_freq,
                       attention_factor, cache, slots):
    rows = qkv.shape[0]
    q = torch.empty(rows, q_heads, head_dim, dtype=torch.bfloat16, device=qkv.device)
    native().ops.qk_norm_rope_cache(
        qkv.data_ptr(), qkv.stride(0), rows, q_heads, kv_heads, head_dim, _ptr(q_norm),
        _ptr(k_norm), float(eps), positions.data_ptr(), inv_freq.data_ptr(),
        float(attention_factor), q.data_ptr(), cache.data_ptr(), slots.data_ptr(), _stream())
    return q


def _attn_common(segments: torch.Tensor) -> None:
    if segments.dtype != torch.int32 or segments.dim() != 2 or segments.shape[1] != 5:
        raise ValueError("segments are int32 [n, 5]: row_start, len, cached, table_start, nblocks")


def paged_decode(q, cache, table, segments, kv_heads, max_keys, scale=None, keys_per_split=2048, out=None,
                 counters=None):
    """Flash-decoding of one-row segments over the paged cache. q: [rows, q_heads, d]. With
    `counters` (int32, zero, one per segment and key/value head) the splits merge in the kernel."""
    _attn_common(segments)
    rows, q_heads, d = q.shape
    out = torch.empty_like(q) if out is None else out
    s = scratch(q.device)
    n = segments.shape[0]
    splits = (max_keys + keys_per_split - 1) // keys_per_split
    need = n * q_heads * splits
    po = torch.empty(need * d if splits > 1 else 1, dtype=torch.float32, device=q.device)
    pl = torch.empty(need if splits > 1 else 1, dtype=torch.float32, device=q.device)
    native().ops.paged_decode(
        q.data_ptr(), out.data_ptr(), cache.data_ptr(), table.data_ptr(), segments.data_ptr(), n,
        q_heads, kv_heads, d, float(scale if scale is not None else d ** -0.5), po.data_ptr(),
        pl.data_ptr(), need, int(max_keys), keys_per_split, s.status.data_ptr(), _stream(),
        0 if counters is None else counters.data_ptr())
    return out


def prefill_work(segments_cpu, group: int) -> torch.Tensor:
    """(segment, query tile) pairs of the prefill kernel, as int32 [n, 2]."""
    work = []
    for i, (_, length, _, _, _) in enumerate(segments_cpu.tolist()):
        for tile in range((length * group + 63) // 64):
            work.append((i, tile))
    return torch.tensor(work, dtype=torch.int32).reshape(-1, 2)


def paged_prefill(q, cache, table, segments, kv_heads, work, scale=None, out=None):
    """Causal attention of segments' rows over their history and themselves."""
    _attn_common(segments)
    rows, q_heads, d = q.shape
    out = torch.empty_like(q) if out is None else out
    s = scratch(q.device)
    native().ops.paged_prefill(
        q.data_ptr(), out.data_ptr(), cache.data_ptr(), table.data_ptr(), segments.data_ptr(),
        segments.shape[0], q_heads, kv_heads, d, float(scale if scale is not None else d ** -0.5),
        work.data_ptr(), work.shape[0], s.status.data_ptr(), _stream())
    return out
