"""The engine's paged decoder call on the host, in FP32 PyTorch.

It runs the same call semantics as the GPU engine (requests of block IDs and cached positions,
one-row requests laid out first, a paged KV cache of 16-token blocks, kept rows returned in
request order) with plain FP32 math and no intermediate rounding. It is the CPU path of small
models and the oracle the GPU engine's plans are checked against.
"""

from __future__ import annotations

import dataclasses

import torch

from . import dense, reference

BLOCK = 16


@dataclasses.dataclass
class Request:
    blocks: list[int]
    cached: int
    tokens: torch.Tensor  # int32 [n]
    keep: str | tuple[int, int] = "last"  # "none" | "last" | "all" | (from, to)


def layout(lengths: list[int]) -> list[tuple[int, int]]:
    """Call rows of each request: one-row requests first, then the others, in request order."""
    spans: list[tuple[int, int]] = [(0, 0)] * len(lengths)
    start = 0
    for one in (True, False):
        for i, n in enumerate(lengths):
            if (n == 1) == one:
                spans[i] = (start, start + n)
                start += n
    return spans


class CpuDecoder:
    """A decoder of engine-layout weights `w` (single chip) on a paged FP32 cache of `blocks`."""

    def __init__(self, cfg: dict, w: dict[str, torch.Tensor], blocks: int):
        self.cfg = cfg
        self.w = {k: v.float() for k, v in w.items()}
        L, kvh, D = cfg["layers"], cfg["kv_heads"], cfg.get("head_dim", 128)
        self.cache = torch.zeros(L, blocks, 2, kvh, BLOCK, D)
        self.freqs = dense.inv_freq(cfg)
        self.gate_up = {}
        for l in range(L):
            g, u = dense.split_gate_up(self.w[f"layers.{l}.gate_up"])
            self.gate_up[l] = (g, u)

    def forward(self, requests: list[Request]) -> torch.Tensor:
        """Logits [kept rows, vocab] of one call."""
        cfg, w = self.cfg, self.w
        H, D = cfg["hidden"], cfg.get("head_dim", 128)
        qh, kvh, eps = cfg["q_heads"], cfg["kv_heads"], cfg["eps"]
        spans = layout([len(r.tokens) for r in requests])
        T = max(e for _, e in spans)
        ids = torch.zeros(T, dtype=torch.long)
        pos = torch.zeros(T, dtype=torch.long)
        for r, (s, e) in zip(requests, spans):
            ids[s:e] = r.tokens.long()
            pos[s:e] = torch.arange(r.cached, r.cached + (e - s))
        x = w["embed"][ids]
        for l in range(cfg["layers"]):
            p = f"layers.{l}."
            h = reference.rmsnorm(x, w[p + "in_norm"], eps)
            qkv = h @ w[p + "qkv"].T
            q, k, v = reference.qk_front(qkv, qh, kvh, D, w.get(p + "q_norm"), w.get(p + "k_norm"), eps, pos,
                                         self.freqs, round_bf16=False)
            # Store the call's keys and values in their slots, then attend each request's history.
            for r, (s, e) in zip(requests, spans):
                for i in range(e - s):
                    position = r.cached + i
                    block = r.blocks[position // BLOCK]
                    self.cache[l, block, 0, :, position % BLOCK] = k[s + i]
                    self.cache[l, block, 1, :, position % BLOCK] = v[s + i]
            att = torch.zeros(T, qh, D)
            for r, (s, e) in zip(requests, spans):
                keys = r.cached + (e - s)
                nb = (keys + BLOCK - 1) // BLOCK
                pages = self.cache[l, r.blocks[:nb]]  # [nb, 2, kvh, 16, D]
                kk = pages[:, 0].permute(0, 2, 1, 3).reshape(nb * BLOCK, kvh, D)[:keys]
                vv = pages[:, 1].permute(0, 2, 1, 3).reshape(nb * BLOCK, kvh, D)[:keys]
                g = qh // kvh
                kk, vv = kk.repeat_interleave(g, 1), vv.repeat_interleave(g, 1)
                sc = torch.einsum("lhd,khd->hlk", q[s:e], kk) * D ** -0.5
                mask = torch.arange(keys)[None, :] <= (torch.arange(e - s)[:, None] + r.cached)
                sc = sc.masked_fill(~mask[None], float("-inf"))
                att[s:e] = torch.einsum("hlk,khd->lhd", torch.softmax(sc, -1), vv)
            x = x + att.reshape(T, qh * D) @ w[p + "o"].T
            h = reference.rmsnorm(x, w[p + "post_norm"], eps)
            gate, up = self.gate_up[l]
            x = x + (torch.nn.functional.silu(h @ gate.T) * (h @ up.T)) @ w[p + "down"].T
        h = reference.rmsnorm(x, w["final_norm"], eps)
        kept: list[int] = []
        for r, (s, e) in zip(requests, spans):
            if r.keep == "last":
                kept.append(e - 1)
            elif r.keep == "all":
                kept.extend(range(s, e))
            elif isinstance(r.keep, tuple):
                kept.extend(range(s + r.keep[0], s + r.keep[1]))
        head = w["lm_head"] if "lm_head" in w else w["embed"]
        return h[kept] @ head[: cfg["vocab"]].T
