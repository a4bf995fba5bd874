"""Named model geometries: the architectures the benchmarks and tests instantiate with synthetic
weights (random-init N(0, 0.02)), matching the published shapes of each checkpoint."""

from __future__ import annotations

import copy

QWEN3_ROPE = {"type": "default", "theta": 1_000_000.0}

CONFIGS: dict[str, dict] = {
    # The tiny Qwen3-architecture decoder of the CPU oracle configuration.
    "tiny-qwen3": dict(
        architecture="Qwen3ForCausalLM", family="qwen3", size="tiny", hidden=256, intermediate=768,
        layers=2, q_heads=4, kv_heads=2, head_dim=64, vocab=1024, eps=1e-6, qk_norm=True, tied=True,
        rope=QWEN3_ROPE, window=4096, rows=8192,
    ),
    # A tiny Qwen3 geometry that splits over 2, 4 and 8 chips (tensor-parallel tests).
    "tiny-qwen3-tp": dict(
        architecture="Qwen3ForCausalLM", family="qwen3", size="tiny", hidden=256, intermediate=1024,
        layers=2, q_heads=8, kv_heads=2, head_dim=64, vocab=1024, eps=1e-6, qk_norm=True, tied=True,
        rope=QWEN3_ROPE, window=4096, rows=8192,
    ),
    # A tiny Qwen3-MoE geometry (16 experts, top-4) for the expert tests; splits over 2/4/8 chips.
    "tiny-qwen3-moe": dict(
        architecture="Qwen3MoeForCausalLM", family="qwen3_moe", size="tiny", hidden=256, intermediate=768,
        layers=2, q_heads=8, kv_heads=2, head_dim=64, vocab=1024, eps=1e-6, qk_norm=True, tied=False,
        rope=QWEN3_ROPE, window=4096, rows=8192, experts=16, top_k=4, expert_intermediate=256,
        norm_topk=True,
    ),
    "qwen3-0.6b": dict(
        architecture="Qwen3ForCausalLM", family="qwen3", size="0.6B", hidden=1024, intermediate=3072,
        layers=28, q_heads=16, kv_heads=8, head_dim=128, vocab=151936, eps=1e-6, qk_norm=True,
        tied=True, rope=QWEN3_ROPE, window=40960, rows=8192,
    ),
    "qwen3-1.7b": dict(
        architecture="Qwen3ForCausalLM", family="qwen3", size="1.7B", hidden=2048, intermediate=6144,
        layers=28, q_heads=16, kv_heads=8, head_dim=128, vocab=151936, eps=1e-6, qk_norm=True,
        tied=True, rope=QWEN3_ROPE, window=40960, rows=8192,
    ),
    "qwen3-4b": dict(
        architecture="Qwen3ForCausalLM", family="qwen3", size="4B", hidden=2560, intermediate=9728,
        layers=36, q_heads=32, kv_heads=8, head_dim=128, vocab=151936, eps=1e-6, qk_norm=True,
        tied=True, rope=QWEN3_ROPE, window=40960, rows=8192,
    ),
    "qwen3-8b": dict(
        architecture="Qwen3ForCausalLM", family="qwen3", size="8B", hidden=4096, intermediate=12288,
        layers=36, q_heads=32, kv_heads=8, head_dim=128, vocab=151936, eps=1e-6, qk_norm=True,
        tied=False, rope=QWEN3_ROPE, window=40960, rows=8192,
    ),
    "llama-3.1-8b": dict(
        architecture="LlamaForCausalLM", family="llama", size="8B", hidden=4096, intermediate=14336,
        layers=32, q_heads=32, kv_heads=8, head_dim=128, vocab=128256, eps=1e-5, qk_norm=False,
        tied=False, window=131072, rows=8192,
        rope={"type": "llama3", "theta": 500000.0, "factor": 8.0, "low_freq_factor": 1.0,
              "high_freq_factor": 4.0, "original_max_positions": 8192},
    ),
    "llama-3.3-70b": dict(
        architecture="LlamaForCausalLM", family="llama", size="70B", hidden=8192, intermediate=28672,
        layers=80, q_heads=64, kv_heads=8, head_dim=128, vocab=128256, eps=1e-5, qk_norm=False,
        tied=False, window=131072, rows=8192,
        rope={"type": "llama3", "theta": 500000.0, "factor": 8.0, "low_freq_factor": 1.0,
              "high_freq_factor": 4.0, "original_max_positions": 8192},
    ),
    "qwen3-30b-a3b": dict(
        architecture="Qwen3MoeForCausalLM", family="qwen3_moe", size="30B-A3B", hidden=2048,
        intermediate=6144, layers=48, q_heads=32, kv_heads=4, head_dim=128, vocab=151936, eps=1e-6,
        qk_norm=True, tied=False, rope=QWEN3_ROPE, window=40960, rows=8192, experts=128, top_k=8,
        expert_intermediate=768, norm_topk=True,
    ),
    # A tiny Mixtral geometry (8 experts, top-2) that splits over 2/4/8 chips.
    "tiny-mixtral": dict(
        architecture="MixtralForCausalLM", family="mixtral", size="tiny", hidden=256, intermediate=256,
        layers=2, q_heads=8, kv_heads=2, head_dim=64, vocab=1024, eps=1e-5, qk_norm=False, tied=False,
        rope={"type": "default", "theta": 1_000_000.0}, window=4096, rows=8192, experts=8, top_k=2,
        expert_intermediate=256, norm_topk=True,
    ),
    "mixtral-8x7b": dict(
        architecture="MixtralForCausalLM", family="mixtral", size="8x7B", hidden=4096, intermediate=14336,
        layers=32, q_heads=32, kv_heads=8, head_dim=128, vocab=32000, eps=1e-5, qk_norm=False, tied=False,
        rope={"type": "default", "theta": 1_000_000.0}, window=32768, rows=8192, experts=8, top_k=2,
        expert_intermediate=14336, norm_topk=True,
    ),
}


# Quantized serving configurations: the same geometries with block-scaled FP8 (W8A8) or NVFP4
# (W4A4 on the block-scaled MMA) projections.
CONFIGS["llama-3.1-8b-fp8"] = dict(CONFIGS["llama-3.1-8b"], precision="float8_e4m3fn", weight_format="fp8_block")
CONFIGS["llama-3.3-70b-nvfp4"] = dict(CONFIGS["llama-3.3-70b"], precision="uint8", weight_format="nvfp4_a4")
CONFIGS["llama-3.1-8b-nvfp4"] = dict(CONFIGS["llama-3.1-8b"], precision="uint8", weight_format="nvfp4_a4")
CONFIGS["qwen3-8b-fp8"] = dict(CONFIGS["qwen3-8b"], precision="float8_e4m3fn", weight_format="fp8_block")
# Mistral NeMo 12B (head_dim 128 below hidden / heads) and its static per-tensor FP8 checkpoint.
CONFIGS["mistral-nemo-12b"] = dict(
    architecture="MistralForCausalLM", family="mistral", size="12B", hidden=5120, intermediate=14336, layers=40,
    q_heads=32, kv_heads=8, head_dim=128, vocab=131072, eps=1e-5, qk_norm=False, tied=False,
    rope={"type": "default", "theta": 1_000_000.0}, window=131072, rows=8192)
CONFIGS["mistral-nemo-12b-fp8"] = dict(CONFIGS["mistral-nemo-12b"], precision="float8_e4m3fn",
                                       weight_format="fp8_static")
CONFIGS["tiny-mistral"] = dict(
    architecture="MistralForCausalLM", family="mistral", size="tiny", hidden=256, intermediate=768, layers=2,
    q_heads=4, kv_heads=2, head_dim=64, vocab=1024, eps=1e-5, qk_norm=False, tied=False,
    rope={"type": "default", "theta": 1_000_000.0}, window=4096, rows=8192)


def get(name: str, **overrides) -> dict:
    cfg = copy.deepcopy(CONFIGS[name])
    cfg.update(overrides)
    return cfg
