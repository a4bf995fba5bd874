"""Dense PyTorch forward of the decoder families on the engine's weight layout: the oracle of the
engine's paged calls (full causal attention over each sequence, FP32 math)."""

from __future__ import annotations

import torch

from . import reference


def split_gate_up(gate_up: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Gate and up rows of the engine's gate/up weight (128-row blocks alternating gate, up)."""
    rows, k = gate_up.shape
    blocks = gate_up.reshape(rows // 256, 2, 128, k)
    return blocks[:, 0].reshape(-1, k), blocks[:, 1].reshape(-1, k)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """The engine's gate/up layout of separate gate [I, K] and up [I, K] weights."""
    i, k = gate.shape
    return torch.stack([gate.reshape(i // 128, 128, k), up.reshape(i // 128, 128, k)], 1).reshape(2 * i, k)


def inv_freq(cfg: dict) -> torch.Tensor:
    d = cfg.get("head_dim", 128)
    rope = cfg.get("rope", {"type": "default", "theta": 10000.0})
    base = 1.0 / (rope.get("theta", 10000.0) ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    kind = rope.get("type", "default")
    if kind == "linear":
        base = base / rope["factor"]
    elif kind == "llama3":
        import math

        old = rope["original_max_positions"]
        low_wl, high_wl = old / rope["low_freq_factor"], old / rope["high_freq_factor"]
        out = base.clone()
        for j, f in enumerate(base.tolist()):
            wl = 2 * math.pi / f
            if wl < high_wl:
                out[j] = f
            elif wl > low_wl:
                out[j] = f / rope["factor"]
            else:
                s = (old / wl - rope["low_freq_factor"]) / (rope["high_freq_factor"] - rope["low_freq_factor"])
                out[j] = (1 - s) * f / rope["factor"] + s * f
        base = out
    return base.float()


def linear(x: torch.Tensor, w) -> torch.Tensor:
    """``x @ w.T`` in FP32 for a BF16 weight, or under a quantized weight's contract."""
    if isinstance(w, torch.Tensor):
        return x @ w.float().T
    return reference.quantized_linear(x, w)


def _gate_up(x: torch.Tensor, w) -> tuple[torch.Tensor, torch.Tensor]:
    full = linear(x, w)
    T = full.shape[0]
    blocks = full.view(T, -1, 2, 128)
    return blocks[:, :, 0].reshape(T, -1), blocks[:, :, 1].reshape(T, -1)


def forward(w: dict, cfg: dict, ids: torch.Tensor, round_bf16: bool = True, head: bool = True) -> torch.Tensor:
    """Logits [len(ids), vocab] of one sequence from position 0, FP32 math; with `round_bf16` every
    stored activation is rounded to BF16 where the engine's GPU kernels store BF16. Without `head`,
    the final-normed hidden rows [len(ids), hidden] (a base model's output)."""
    rb = (lambda t: t.bfloat16().float()) if round_bf16 else (lambda t: t)
    H, D = cfg["hidden"], cfg.get("head_dim", 128)
    qh, kvh = cfg["q_heads"], cfg["kv_heads"]
    eps = cfg["eps"]
    T = ids.shape[0]
    x = w["embed"][ids.long()].float()
    pos = torch.arange(T)
    freqs = inv_freq(cfg)
    mask = torch.ones(T, T, dtype=torch.bool).tril()
    for l in range(cfg["layers"]):
        p = f"layers.{l}."
        h = rb(reference.rmsnorm(x, w[p + "in_norm"], eps))
        qkv = rb(linear(h, w[p + "qkv"]))
        q, k, v = reference.qk_front(qkv, qh, kvh, D, w.get(p + "q_norm"), w.get(p + "k_norm"), eps, pos,
                                     freqs, round_bf16=round_bf16)
        q, k = rb(q), rb(k)
        g = qh // kvh
        k = k.repeat_interleave(g, 1)
        v = v.repeat_interleave(g, 1)
        s = torch.einsum("qhd,khd->hqk", q, k) * D ** -0.5
        s = s.masked_fill(~mask[None], float("-inf"))
        a = rb(torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(T, qh * D))
        x = rb(x + linear(a, w[p + "o"]))
        h = rb(reference.rmsnorm(x, w[p + "post_norm"], eps))
        if cfg.get("experts", 0):
            E, I = cfg["experts"], cfg["expert_intermediate"]
            moe = reference.moe_forward(h.bfloat16(), w[p + "router"].bfloat16(),
                                        w[p + "experts_gate_up"].bfloat16().view(E, 2 * I, H),
                                        w[p + "experts_down"].bfloat16().view(E, H, I), cfg["top_k"],
                                        cfg.get("norm_topk", True))
            x = rb(x + moe.float())
            continue
        g, u = _gate_up(h, w[p + "gate_up"])
        act = rb(reference.swiglu(g, u)) if round_bf16 else torch.nn.functional.silu(g) * u
        x = rb(x + linear(act, w[p + "down"]))
    h = rb(reference.rmsnorm(x, w["final_norm"], eps))
    if not head:
        return h
    out = w["lm_head"] if "lm_head" in w else w["embed"]
    return h @ out[: cfg["vocab"]].float().T
