"""Synthetic Hugging Face checkpoints: a config.json and safetensors files of random-init
N(0, std) weights under the HF tensor names of a named geometry. Tests and benchmarks load them
through the public LoadOptions path (there is no network for published checkpoints)."""

from __future__ import annotations

import json
import os

import torch

from . import configs


def hf_config(cfg: dict) -> dict:
    """The HF config.json of an engine geometry."""
    out = {
        "architectures": [cfg["architecture"]],
        "model_type": {"qwen3": "qwen3", "llama": "llama", "mistral": "mistral", "qwen3_moe": "qwen3_moe",
                       "mixtral": "mixtral"}[cfg["family"]],
        "hidden_size": cfg["hidden"],
        "intermediate_size": cfg["intermediate"],
        "num_hidden_layers": cfg["layers"],
        "num_attention_heads": cfg["q_heads"],
        "num_key_value_heads": cfg["kv_heads"],
        "head_dim": cfg["head_dim"],
        "vocab_size": cfg["vocab"],
        "rms_norm_eps": cfg["eps"],
        "tie_word_embeddings": cfg["tied"],
        "max_position_embeddings": cfg["window"],
        "torch_dtype": "bfloat16",
        "attention_bias": False,
    }
    rope = cfg.get("rope", {"type": "default", "theta": 10000.0})
    out["rope_theta"] = rope["theta"]
    if rope.get("type", "default") != "default":
        scaling = {"rope_type": rope["type"], "factor": rope["factor"]}
        for k in ("low_freq_factor", "high_freq_factor"):
            if k in rope:
                scaling[k] = rope[k]
        if "original_max_positions" in rope:
            scaling["original_max_position_embeddings"] = rope["original_max_positions"]
        out["rope_scaling"] = scaling
    if cfg["family"] == "qwen3":
        out["use_sliding_window"] = False
    if cfg["family"] == "mixtral":
        out.update(num_local_experts=cfg["experts"], num_experts_per_tok=cfg["top_k"],
                   intermediate_size=cfg["expert_intermediate"], sliding_window=None, router_jitter_noise=0.0)
    if cfg["family"] == "qwen3_moe":
        out.update(num_experts=cfg["experts"], num_experts_per_tok=cfg["top_k"],
                   moe_intermediate_size=cfg["expert_intermediate"], norm_topk_prob=cfg["norm_topk"],
                   decoder_sparse_step=1, mlp_only_layers=[])
    return out


# HF names of a mixture-of-experts block: (prefix under the layer, gate, up, down projections).
MOE_NAMES = {"qwen3_moe": ("mlp.", "gate_proj", "up_proj", "down_proj"),
             "mixtral": ("block_sparse_moe.", "w1", "w3", "w2")}


def hf_weights(cfg: dict, seed: int = 0, std: float = 0.02) -> dict[str, torch.Tensor]:
    """HF-named BF16 weights of a geometry (CPU tensors)."""
    g = torch.Generator().manual_seed(seed)
    H, D, I = cfg["hidden"], cfg["head_dim"], cfg["intermediate"]
    qh, kvh, V = cfg["q_heads"], cfg["kv_heads"], cfg["vocab"]

    def rnd(*shape):
        return (torch.randn(*shape, generator=g) * std).bfloat16()

    def ones(n):
        return (1.0 + 0.1 * torch.randn(n, generator=g)).bfloat16()

    w = {"model.embed_tokens.weight": rnd(V, H), "model.norm.weight": ones(H)}
    if not cfg["tied"]:
        w["lm_head.weight"] = rnd(V, H)
    for l in range(cfg["layers"]):
        p = f"model.layers.{l}."
        w[p + "input_layernorm.weight"] = ones(H)
        w[p + "post_attention_layernorm.weight"] = ones(H)
        w[p + "self_attn.q_proj.weight"] = rnd(qh * D, H)
        w[p + "self_attn.k_proj.weight"] = rnd(kvh * D, H)
        w[p + "self_attn.v_proj.weight"] = rnd(kvh * D, H)
        w[p + "self_attn.o_proj.weight"] = rnd(H, qh * D)
        if cfg.get("qk_norm"):
            w[p + "self_attn.q_norm.weight"] = ones(D)
            w[p + "self_attn.k_norm.weight"] = ones(D)
        if cfg["family"] in MOE_NAMES:
            E, Ie = cfg["experts"], cfg["expert_intermediate"]
            block, gname, uname, dname = MOE_NAMES[cfg["family"]]
            w[p + block + "gate.weight"] = rnd(E, H)
            for e in range(E):
                w[p + f"{block}experts.{e}.{gname}.weight"] = rnd(Ie, H)
                w[p + f"{block}experts.{e}.{uname}.weight"] = rnd(Ie, H)
                w[p + f"{block}experts.{e}.{dname}.weight"] = rnd(H, Ie)
        else:
            w[p + "mlp.gate_proj.weight"] = rnd(I, H)
            w[p + "mlp.up_proj.weight"] = rnd(I, H)
            w[p + "mlp.down_proj.weight"] = rnd(H, I)
    return w


def write(directory: str, name_or_cfg, seed: int = 0, std: float = 0.02, shards: int = 1) -> dict:
    """Writes a synthetic checkpoint of `name_or_cfg` into `directory`; returns its weights."""
    from safetensors.torch import save_file

    cfg = configs.get(name_or_cfg) if isinstance(name_or_cfg, str) else name_or_cfg
    os.makedirs(directory, exist_ok=True)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(hf_config(cfg), f)
    weights = hf_weights(cfg, seed, std)
    names = sorted(weights)
    if shards == 1:
        save_file(weights, os.path.join(directory, "model.safetensors"))
    else:
        per = (len(names) + shards - 1) // shards
        weight_map = {}
        for s in range(shards):
            part = names[s * per : (s + 1) * per]
            fname = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
            save_file({n: weights[n] for n in part}, os.path.join(directory, fname))
            weight_map.update({n: fname for n in part})
        with open(os.path.join(directory, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {}, "weight_map": weight_map}, f)
    return weights


def engine_weights(cfg: dict, hf: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """The engine's (single-chip) weight layout of HF-named weights, for the dense oracle."""
    from .dense import interleave_gate_up

    out = {"embed": hf["model.embed_tokens.weight"], "final_norm": hf["model.norm.weight"]}
    if "lm_head.weight" in hf:
        out["lm_head"] = hf["lm_head.weight"]
    for l in range(cfg["layers"]):
        p, e = f"model.layers.{l}.", f"layers.{l}."
        out[e + "in_norm"] = hf[p + "input_layernorm.weight"]
        out[e + "post_norm"] = hf[p + "post_attention_layernorm.weight"]
        out[e + "qkv"] = torch.cat([hf[p + "self_attn.q_proj.weight"], hf[p + "self_attn.k_proj.weight"],
                                    hf[p + "self_attn.v_proj.weight"]])
        out[e + "o"] = hf[p + "self_attn.o_proj.weight"]
        if p + "self_attn.q_norm.weight" in hf:
            out[e + "q_norm"] = hf[p + "self_attn.q_norm.weight"]
            out[e + "k_norm"] = hf[p + "self_attn.k_norm.weight"]
        if p + "mlp.gate_proj.weight" in hf:
            out[e + "gate_up"] = interleave_gate_up(hf[p + "mlp.gate_proj.weight"], hf[p + "mlp.up_proj.weight"])
            out[e + "down"] = hf[p + "mlp.down_proj.weight"]
        if cfg.get("experts"):
            E = cfg["experts"]
            block, gname, uname, dname = MOE_NAMES[cfg["family"]]
            q = p + block
            out[e + "router"] = hf[q + "gate.weight"]
            out[e + "experts_gate_up"] = torch.cat([
                interleave_gate_up(hf[q + f"experts.{x}.{gname}.weight"], hf[q + f"experts.{x}.{uname}.weight"])
                for x in range(E)])
            out[e + "experts_down"] = torch.cat([hf[q + f"experts.{x}.{dname}.weight"] for x in range(E)])
    return out


LORA_MODULES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def write_lora(directory: str, cfg: dict, r: int = 8, alpha: float = 16.0, seed: int = 0, std: float = 0.05,
               modules=LORA_MODULES) -> dict[str, torch.Tensor]:
    """A synthetic PEFT LoRA checkpoint for a geometry (adapter_config.json and
    adapter_model.safetensors); returns {"<layer>.<module>": (A [r, in], B [out, r])}."""
    from safetensors.torch import save_file

    os.makedirs(directory, exist_ok=True)
    g = torch.Generator().manual_seed(seed)
    H, D, I = cfg["hidden"], cfg["head_dim"], cfg["intermediate"]
    shapes = {"q_proj": (H, cfg["q_heads"] * D), "k_proj": (H, cfg["kv_heads"] * D),
              "v_proj": (H, cfg["kv_heads"] * D), "o_proj": (cfg["q_heads"] * D, H),
              "gate_proj": (H, I), "up_proj": (H, I), "down_proj": (I, H)}
    tensors, out = {}, {}
    for l in range(cfg["layers"]):
        for m in modules:
            fin, fout = shapes[m]
            a = (torch.randn(r, fin, generator=g) * std).bfloat16()
            b = (torch.randn(fout, r, generator=g) * std).bfloat16()
            path = ("self_attn." if m in ("q_proj", "k_proj", "v_proj", "o_proj") else "mlp.") + m
            tensors[f"base_model.model.model.layers.{l}.{path}.lora_A.weight"] = a
            tensors[f"base_model.model.model.layers.{l}.{path}.lora_B.weight"] = b
            out[f"{l}.{m}"] = (a, b)
    save_file(tensors, os.path.join(directory, "adapter_model.safetensors"))
    config = {"r": r, "lora_alpha": alpha, "target_modules": list(modules), "bias": "none",
              "peft_type": "LORA", "use_dora": False, "use_rslora": False}
    with open(os.path.join(directory, "adapter_config.json"), "w") as f:
        json.dump(config, f)
    return out


def merge_lora(weights: dict, cfg: dict, lora: dict, r: int, alpha: float) -> dict:
    """Engine-layout FP32 weights with a LoRA update merged (W + alpha / r * B A), for the dense
    oracle."""
    from .dense import interleave_gate_up, split_gate_up

    scale = alpha / r
    out = dict(weights)
    H, D = cfg["hidden"], cfg["head_dim"]
    qr, kvr = cfg["q_heads"] * D, cfg["kv_heads"] * D
    for l in range(cfg["layers"]):
        def delta(m):
            a, b = lora[f"{l}.{m}"]
            return (b.float() * scale).bfloat16().float() @ a.float()
        p = f"layers.{l}."
        qkv = out[p + "qkv"].float().clone()
        qkv[:qr] += delta("q_proj")
        qkv[qr:qr + kvr] += delta("k_proj")
        qkv[qr + kvr:] += delta("v_proj")
        out[p + "qkv"] = qkv
        out[p + "o"] = out[p + "o"].float() + delta("o_proj")
        gate, up = split_gate_up(out[p + "gate_up"].float())
        out[p + "gate_up"] = interleave_gate_up(gate + delta("gate_proj"), up + delta("up_proj"))
        out[p + "down"] = out[p + "down"].float() + delta("down_proj")
    return out


def gemma4_unified_config(text: int = 256, embed: int = 192, positions: int = 40, samples: int = 640,
                          patch_size: int = 16, pooling: int = 3, eps: float = 1e-6) -> dict:
    """A Gemma-4 unified config.json of the given media-encoder widths (the published model:
    text 3840, embed 3840, positions 1120, samples 640)."""
    return {
        "architectures": ["Gemma4UnifiedForConditionalGeneration"],
        "model_type": "gemma4_unified",
        "text_config": {"hidden_size": text},
        "vision_config": {"mm_embed_dim": embed, "mm_posemb_size": positions, "patch_size": patch_size,
                          "pooling_kernel_size": pooling, "rms_norm_eps": eps},
        "audio_config": {"audio_embed_dim": samples, "rms_norm_eps": eps},
    }


def write_gemma4_encoder(directory: str, config: dict, seed: int = 0, std: float = 0.05) -> dict:
    """A synthetic Gemma-4 unified checkpoint: the media embedders under `model.` (and one language
    model tensor, which a load of the encoder alone ignores); returns the embedders' tensors."""
    from safetensors.torch import save_file

    os.makedirs(directory, exist_ok=True)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(config, f)
    v = config["vision_config"]
    E, T, S, N = v["mm_embed_dim"], config["text_config"]["hidden_size"], config["audio_config"]["audio_embed_dim"], v["mm_posemb_size"]
    P = 3 * (v["patch_size"] * v["pooling_kernel_size"]) ** 2
    g = torch.Generator().manual_seed(seed)

    def rnd(*shape, scale=std, mean=0.0):
        return (torch.randn(*shape, generator=g) * scale + mean).bfloat16()

    e = "model.vision_embedder."
    w = {
        e + "patch_ln1.weight": rnd(P, scale=0.1, mean=1.0), e + "patch_ln1.bias": rnd(P, scale=0.1),
        e + "patch_dense.weight": rnd(E, P), e + "patch_dense.bias": rnd(E, scale=0.1),
        e + "patch_ln2.weight": rnd(E, scale=0.1, mean=1.0), e + "patch_ln2.bias": rnd(E, scale=0.1),
        e + "pos_embedding": rnd(N, 2, E, scale=0.5),
        e + "pos_norm.weight": rnd(E, scale=0.1, mean=1.0), e + "pos_norm.bias": rnd(E, scale=0.1),
        "model.embed_vision.embedding_projection.weight": rnd(T, E),
        "model.embed_audio.embedding_projection.weight": rnd(T, S),
    }
    save_file({**w, "model.language_model.embed_tokens.weight": rnd(8, T)}, os.path.join(directory, "model.safetensors"))
    return w


def write_tokenizer(directory: str, vocab: int) -> None:
    """A word-level tokenizer of `vocab` tokens named t0, t1, ... (whitespace-separated), saved
    beside a synthetic checkpoint for frameworks that open a tokenizer even when prompts come as
    token IDs."""
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    tok = Tokenizer(models.WordLevel(vocab={f"t{i}": i for i in range(vocab)}, unk_token="t0"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="t0", pad_token="t1", eos_token="t2").save_pretrained(directory)


def hf_shapes(cfg: dict) -> dict[str, tuple[int, ...]]:
    """The HF names and shapes `hf_weights` writes for a geometry, without allocating them."""
    H, D, I = cfg["hidden"], cfg["head_dim"], cfg["intermediate"]
    qh, kvh, V = cfg["q_heads"], cfg["kv_heads"], cfg["vocab"]
    out = {"model.embed_tokens.weight": (V, H), "model.norm.weight": (H,)}
    if not cfg["tied"]:
        out["lm_head.weight"] = (V, H)
    for l in range(cfg["layers"]):
        p = f"model.layers.{l}."
        out[p + "input_layernorm.weight"] = (H,)
        out[p + "post_attention_layernorm.weight"] = (H,)
        out[p + "self_attn.q_proj.weight"] = (qh * D, H)
        out[p + "self_attn.k_proj.weight"] = (kvh * D, H)
        out[p + "self_attn.v_proj.weight"] = (kvh * D, H)
        out[p + "self_attn.o_proj.weight"] = (H, qh * D)
        if cfg.get("qk_norm"):
            out[p + "self_attn.q_norm.weight"] = (D,)
            out[p + "self_attn.k_norm.weight"] = (D,)
        if cfg["family"] in MOE_NAMES:
            E, Ie = cfg["experts"], cfg["expert_intermediate"]
            block, gname, uname, dname = MOE_NAMES[cfg["family"]]
            out[p + block + "gate.weight"] = (E, H)
            for e in range(E):
                out[p + f"{block}experts.{e}.{gname}.weight"] = (Ie, H)
                out[p + f"{block}experts.{e}.{uname}.weight"] = (Ie, H)
                out[p + f"{block}experts.{e}.{dname}.weight"] = (H, Ie)
        else:
            out[p + "mlp.gate_proj.weight"] = (I, H)
            out[p + "mlp.up_proj.weight"] = (I, H)
            out[p + "mlp.down_proj.weight"] = (H, I)
    return out


# The quantization declaration of a static per-tensor FP8 checkpoint (Mistral NeMo FP8 style).
STATIC_FP8 = {"quant_method": "fp8", "activation_scheme": "static"}


def quantize_static_fp8(hf: dict[str, torch.Tensor], amax_in: float = 4.0) -> dict[str, torch.Tensor]:
    """HF-named BF16 weights as a static per-tensor FP8 checkpoint: each projection's E4M3 codes
    of w / weight_scale (weight_scale = amax / 448), its FP32 weight_scale and a calibrated
    input_scale (`amax_in` / 448); other tensors unchanged."""
    out = {}
    for name, w in hf.items():
        if not name.endswith("_proj.weight"):
            out[name] = w
            continue
        base = name[: -len(".weight")]
        scale = max(float(w.float().abs().max()), 1e-12) / 448.0
        out[name] = (w.float() / scale).to(torch.float8_e4m3fn)
        out[base + ".weight_scale"] = torch.tensor(scale, dtype=torch.float32)
        out[base + ".input_scale"] = torch.tensor(amax_in / 448.0, dtype=torch.float32)
    return out


def dequantize_static_fp8(q: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """The BF16 weights a static FP8 checkpoint restores: bf16(code * weight_scale)."""
    out = {}
    for name, t in q.items():
        if name.endswith(".weight_scale") or name.endswith(".input_scale"):
            continue
        if t.dtype == torch.float8_e4m3fn:
            out[name] = (t.float() * q[name[: -len(".weight")] + ".weight_scale"]).bfloat16()
        else:
            out[name] = t
    return out


def write_declared(directory: str, name_or_cfg) -> dict[str, tuple[int, ...]]:
    """A checkpoint of the geometry's full size that holds only headers: config.json and a
    safetensors file whose header declares every tensor (offsets as if the data followed) but
    stores no data, for `Checkpoint.declared` (loading checks of models too large to write).
    Returns the declared shapes."""
    cfg = configs.get(name_or_cfg) if isinstance(name_or_cfg, str) else name_or_cfg
    os.makedirs(directory, exist_ok=True)
    fmt = cfg.get("weight_format", "bf16")
    conf = hf_config(cfg)
    # Quantized geometries declare the published checkpoints' formats: FP8 E4M3 projections with
    # an FP32 scale per 128x128 block, or ModelOpt NVFP4 (packed E2M1 codes, an E4M3 scale per 16
    # inputs, FP32 tensor and input scales). Norms, embedding and head stay BF16.
    if fmt == "fp8_block":
        conf["quantization_config"] = {"quant_method": "fp8", "activation_scheme": "dynamic",
                                       "weight_block_size": [128, 128]}
    elif fmt in ("nvfp4", "nvfp4_a4"):
        conf["quantization_config"] = {"quant_method": "modelopt", "quant_algo": "NVFP4", "group_size": 16}
    elif fmt == "fp8_static":
        conf["quantization_config"] = STATIC_FP8
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(conf, f)
    shapes = dict(hf_shapes(cfg))
    dtypes = {name: "BF16" for name in shapes}
    if fmt != "bf16":
        for name in [n for n in shapes if n.endswith("_proj.weight")]:
            R, C = shapes[name]
            base = name[: -len(".weight")]
            if fmt == "fp8_block":
                dtypes[name] = "F8_E4M3"
                shapes[base + ".weight_scale_inv"] = (-(-R // 128), -(-C // 128))
                dtypes[base + ".weight_scale_inv"] = "F32"
            elif fmt == "fp8_static":
                dtypes[name] = "F8_E4M3"
                for s in ("weight_scale", "input_scale"):
                    shapes[f"{base}.{s}"], dtypes[f"{base}.{s}"] = (), "F32"
            else:
                shapes[name], dtypes[name] = (R, C // 2), "U8"
                shapes[base + ".weight_scale"], dtypes[base + ".weight_scale"] = (R, C // 16), "F8_E4M3"
                for s in ("weight_scale_2", "input_scale"):
                    shapes[f"{base}.{s}"], dtypes[f"{base}.{s}"] = (), "F32"
    write_headers(directory, shapes, dtypes)
    return shapes


def write_headers(directory: str, shapes: dict, dtypes: dict | None = None) -> None:
    """Writes `model.safetensors` holding only a header that declares `shapes` (BF16 unless
    `dtypes` names another type), offsets as if the data followed."""
    import struct

    size = {"BF16": 2, "F32": 4, "F8_E4M3": 1, "U8": 1}
    dtypes = dtypes or {}
    header, at = {}, 0
    for name in sorted(shapes):
        dt = dtypes.get(name, "BF16")
        n = size[dt]
        for d in shapes[name]:
            n *= d
        header[name] = {"dtype": dt, "shape": list(shapes[name]), "data_offsets": [at, at + n]}
        at += n
    raw = json.dumps(header).encode()
    raw += b" " * (-len(raw) % 8)
    with open(os.path.join(directory, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(raw)) + raw)
