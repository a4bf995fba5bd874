"""Plain PyTorch FP32 math of the decoder ops: the oracle every kernel and the engine's CPU path
are checked against.

Each function states the numerical contract of the reference op it restates:
RMSNorm (`ops/normalization/rms_norm.rs:15-20`), RoPE with half-split pairs (`ops/rotary.rs:55-57`),
SwiGLU with SiLU(gate) rounded before the product (`ops/swiglu/mod.rs:1-3`).
"""

from __future__ import annotations

import torch


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """FP32 statistics, FP32 product with the weight, no intermediate rounding."""
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()


def rope(x: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor, factor: float = 1.0) -> torch.Tensor:
    """Rotates pairs (j, j + d/2) of the last axis by ``position * inv_freq[j]``.

    ``x`` is [rows, heads, d] and ``positions`` [rows]."""
    angle = positions.float()[:, None] * inv_freq.float()[None, :]
    cos = (torch.cos(angle) * factor)[:, None, :]
    sin = (torch.sin(angle) * factor)[:, None, :]
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def qk_front(qkv, q_heads, kv_heads, head_dim, q_norm, k_norm, eps, positions, inv_freq, factor=1.0,
             round_bf16=True):
    """Splits packed q/k/v rows, applies the per-head norm and RoPE to q and k.

    With ``round_bf16`` the norm's output is rounded to BF16 before the rotation, as the kernel
    stores it."""
    rows = qkv.shape[0]
    q = qkv[:, : q_heads * head_dim].reshape(rows, q_heads, head_dim).float()
    k = qkv[:, q_heads * head_dim : (q_heads + kv_heads) * head_dim].reshape(rows, kv_heads, head_dim).float()
    v = qkv[:, (q_heads + kv_heads) * head_dim :].reshape(rows, kv_heads, head_dim).float()
    if q_norm is not None:
        q = rmsnorm(q, q_norm, eps)
        k = rmsnorm(k, k_norm, eps)
        if round_bf16:
            q = q.bfloat16().float()
            k = k.bfloat16().float()
    return rope(q, positions, inv_freq, factor), rope(k, positions, inv_freq, factor), v


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``bf16(silu(bf16 gate)) * bf16 up`` in FP32."""
    g = gate.bfloat16().float()
    return torch.nn.functional.silu(g).bfloat16().float() * up.bfloat16().float()


def gather_kv(cache: torch.Tensor, table, table_start: int, keys: int):
    """K and V [keys, kv_heads, d] of one sequence from a paged layer ``cache``
    [blocks, 2, kv_heads, 16, d]."""
    nb = (keys + 15) // 16
    ids = [int(x) for x in table[table_start : table_start + nb]]
    pages = cache[ids]  # [nb, 2, H, 16, d]
    k = pages[:, 0].permute(0, 2, 1, 3).reshape(nb * 16, cache.shape[2], cache.shape[4])[:keys]
    v = pages[:, 1].permute(0, 2, 1, 3).reshape(nb * 16, cache.shape[2], cache.shape[4])[:keys]
    return k.float(), v.float()


def paged_attention(q: torch.Tensor, cache: torch.Tensor, table, segments, scale: float | None = None):
    """Causal GQA attention of every segment's rows over its paged history, in FP32.

    ``q`` [rows, q_heads, d]; ``segments`` rows of (row_start, len, cached, table_start, nblocks).
    Row i of a segment is position cached + i and attends keys 0..cached + i."""
    rows, q_heads, d = q.shape
    kv_heads = cache.shape[2]
    group = q_heads // kv_heads
    scale = d ** -0.5 if scale is None else scale
    out = torch.zeros(rows, q_heads, d, dtype=torch.float32)
    for row_start, length, cached, table_start, _ in [tuple(int(x) for x in s) for s in segments]:
        keys = cached + length
        k, v = gather_kv(cache, table, table_start, keys)
        k = k.repeat_interleave(group, dim=1)  # [keys, q_heads, d]
        v = v.repeat_interleave(group, dim=1)
        qs = q[row_start : row_start + length].float()  # [len, q_heads, d]
        s = torch.einsum("lhd,khd->hlk", qs, k) * scale
        pos = torch.arange(length)[:, None] + cached
        mask = torch.arange(keys)[None, :] <= pos
        s = s.masked_fill(~mask[None], float("-inf"))
        out[row_start : row_start + length] = torch.einsum("hlk,khd->lhd", torch.softmax(s, -1), v)
    return out
