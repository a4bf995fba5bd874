"""The library baseline of the serving benchmark: the same decoder and workload written with stock
PyTorch on the GPU (cuBLAS GEMMs through ``torch.matmul``, PyTorch's fused scaled-dot-product
attention over a contiguous KV cache, NCCL all-reduce for tensor parallelism), eager, no engine
kernels. It is the NCCL + cuBLAS reference point the engine's fused paths are measured against.

Weights are random N(0, std) of the named geometry, sharded like the engine's: q/k/v and gate/up
by columns (heads, intermediate), o and down by rows, followed by an all-reduce.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


class Baseline:
    def __init__(self, cfg: dict, tp: int = 1, rank: int = 0, std: float = 0.02, seed: int = 0):
        self.cfg, self.tp, self.rank = cfg, tp, rank
        H, D = cfg["hidden"], cfg.get("head_dim", 128)
        qh, kvh, inter, V = cfg["q_heads"], cfg["kv_heads"], cfg["intermediate"], cfg["vocab"]
        self.qh, self.kvh = qh // tp, max(kvh // tp, 1)
        self.inter = inter // tp
        self.D, self.H = D, H
        g = torch.Generator(device="cuda").manual_seed(seed + rank)

        def rnd(*shape):
            return (torch.randn(*shape, generator=g, device="cuda") * std).bfloat16()

        self.embed = rnd(V, H)
        self.head = self.embed if cfg["tied"] else rnd(V, H)
        self.layers = []
        for _ in range(cfg["layers"]):
            self.layers.append(dict(
                qkv=rnd((self.qh + 2 * self.kvh) * D, H), o=rnd(H, self.qh * D),
                gate_up=rnd(2 * self.inter, H), down=rnd(H, self.inter),
                n1=torch.ones(H, device="cuda", dtype=torch.bfloat16),
                n2=torch.ones(H, device="cuda", dtype=torch.bfloat16),
                qn=torch.ones(D, device="cuda", dtype=torch.bfloat16) if cfg.get("qk_norm") else None,
                kn=torch.ones(D, device="cuda", dtype=torch.bfloat16) if cfg.get("qk_norm") else None))
        self.norm = torch.ones(H, device="cuda", dtype=torch.bfloat16)
        theta = cfg.get("rope", {}).get("theta", 10000.0)
        self.inv_freq = 1.0 / (theta ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D))
        self.k_cache = self.v_cache = None

    def allocate(self, batch: int, length: int) -> None:
        shape = (len(self.layers), batch, self.kvh, length, self.D)
        self.k_cache = torch.empty(shape, device="cuda", dtype=torch.bfloat16)
        self.v_cache = torch.empty(shape, device="cuda", dtype=torch.bfloat16)

    def _rope(self, x, pos):
        f = pos.float()[:, None] * self.inv_freq[None, :]
        cos, sin = f.cos()[None, None], f.sin()[None, None]
        x1, x2 = x[..., : self.D // 2].float(), x[..., self.D // 2:].float()
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1).bfloat16()

    def _allreduce(self, x):
        if self.tp > 1:
            import torch.distributed as dist

            dist.all_reduce(x)
        return x

    @torch.inference_mode()
    def forward(self, ids: torch.Tensor, start: int, b0: int = 0) -> torch.Tensor:
        """ids [B, T] of sequences b0..b0+B-1 at positions start..start+T-1; greedy next tokens [B]."""
        B, T = ids.shape
        eps = self.cfg["eps"]
        x = F.embedding(ids, self.embed)
        pos = torch.arange(start, start + T, device="cuda")
        for li, w in enumerate(self.layers):
            h = F.rms_norm(x, (self.H,), w["n1"], eps)
            qkv = h @ w["qkv"].T
            q, k, v = qkv.split([self.qh * self.D, self.kvh * self.D, self.kvh * self.D], -1)
            q = q.view(B, T, self.qh, self.D).transpose(1, 2)
            k = k.view(B, T, self.kvh, self.D).transpose(1, 2)
            v = v.view(B, T, self.kvh, self.D).transpose(1, 2)
            if w["qn"] is not None:
                q = F.rms_norm(q, (self.D,), w["qn"], eps)
                k = F.rms_norm(k, (self.D,), w["kn"], eps)
            q, k = self._rope(q, pos), self._rope(k, pos)
            self.k_cache[li, b0:b0 + B, :, start:start + T] = k
            self.v_cache[li, b0:b0 + B, :, start:start + T] = v
            kc, vc = self.k_cache[li, b0:b0 + B, :, : start + T], self.v_cache[li, b0:b0 + B, :, : start + T]
            a = F.scaled_dot_product_attention(q, kc, vc, is_causal=T > 1, enable_gqa=True)
            a = a.transpose(1, 2).reshape(B, T, self.qh * self.D)
            x = x + self._allreduce(a @ w["o"].T)
            h = F.rms_norm(x, (self.H,), w["n2"], eps)
            gu = h @ w["gate_up"].T
            gate, up = gu.split([self.inter, self.inter], -1)
            x = x + self._allreduce((F.silu(gate) * up) @ w["down"].T)
        h = F.rms_norm(x[:, -1], (self.H,), self.norm, eps)
        logits = h @ self.head.T
        return logits.argmax(-1)
