"""The engine's KV layout in vLLM's terms: one full-attention group per layer, 16-token pages of
K then V for this rank's key/value heads in BF16, so vLLM's block IDs are the engine's pool
blocks (engine page = vLLM page size)."""

from __future__ import annotations

import torch

BLOCK = 16
# A layer's page holds K[kv_heads][16][head] then V[kv_heads][16][head]: heads outermost, in vLLM's
# naming the "HND" layout. It is the engine's fixed layout, so it is the only one offered.
LAYOUTS = ("HND",)


def spec(model, model_config) -> dict:
    from vllm.v1.kv_cache_interface import FullAttentionSpec

    g = model.geometry
    pool = model.cache.pools[0]
    heads, head = g["kv_heads"], pool.bytes // (2 * BLOCK * g["kv_heads"] * 2)
    layers = model.cache.groups[0].layers
    n = len(range(*layers)) if isinstance(layers, tuple) else len(layers)
    s = FullAttentionSpec(block_size=BLOCK, num_kv_heads=heads, head_size=head, dtype=torch.bfloat16)
    return {f"model.layers.{i}.self_attn.attn": s for i in range(n)}
