"""Catalog compositions (encoders, encoder-decoders, contrastive, recurrent, hybrid, further
decoders, vision-language): built from config.json alone and checked strictly against checkpoint
headers. The oracle of every name and shape is the transformers module of the same config, built on
the meta device (no values); the checkpoints hold only safetensors headers (`Checkpoint.declared`).
Where transformers keeps routed experts as one 3-D tensor, the oracle splits it into the per-expert
matrices that the published checkpoints store."""

import json
import re

import pytest

import furiosa_opt_engine as engine
from furiosa_opt_models_b200.models import catalog, synthetic

transformers = pytest.importorskip("transformers")
torch = pytest.importorskip("torch")

_IDS = dict(pad_token_id=0, bos_token_id=1, eos_token_id=2)


def _family_configs():
    t = transformers
    bert = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, intermediate_size=128, vocab_size=100,
                max_position_embeddings=40)
    clip_text = dict(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                     vocab_size=100, max_position_embeddings=20)
    clip_vision = dict(hidden_size=48, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
                       image_size=32, patch_size=8)
    llama = dict(hidden_size=64, num_hidden_layers=2, vocab_size=100, num_attention_heads=4, num_key_value_heads=2,
                 intermediate_size=128)
    return {
        "bert": (lambda: t.BertConfig(**bert), t.BertModel),
        "bert_mlm": (lambda: t.BertConfig(**bert), t.BertForMaskedLM),
        "bert_seq": (lambda: t.BertConfig(**bert, num_labels=3), t.BertForSequenceClassification),
        "bert_tok": (lambda: t.BertConfig(**bert, num_labels=5), t.BertForTokenClassification),
        "xlm_roberta": (lambda: t.XLMRobertaConfig(**dict(bert, max_position_embeddings=42)), t.XLMRobertaModel),
        "xlm_roberta_rerank": (lambda: t.XLMRobertaConfig(**dict(bert, max_position_embeddings=42), num_labels=1),
                               t.XLMRobertaForSequenceClassification),
        "clip": (lambda: t.CLIPConfig(text_config=clip_text, vision_config=clip_vision, projection_dim=40),
                 t.CLIPModel),
        "clip_text": (lambda: t.CLIPTextConfig(**clip_text, projection_dim=40), t.CLIPTextModelWithProjection),
        "clip_vision": (lambda: t.CLIPVisionConfig(**clip_vision, projection_dim=40), t.CLIPVisionModelWithProjection),
        "clip_text_plain": (lambda: t.CLIPTextConfig(**clip_text), t.CLIPTextModel),
        "siglip": (lambda: t.SiglipConfig(text_config=clip_text, vision_config=clip_vision), t.SiglipModel),
        "siglip_vision": (lambda: t.SiglipVisionConfig(**clip_vision), t.SiglipVisionModel),
        "t5": (lambda: t.T5Config(d_model=64, d_kv=16, d_ff=128, num_heads=4, num_layers=2, num_decoder_layers=3,
                                  vocab_size=100, feed_forward_proj="relu"), t.T5ForConditionalGeneration),
        "t5_gated_untied": (lambda: t.T5Config(d_model=64, d_kv=8, d_ff=96, num_heads=6, num_layers=1, vocab_size=100,
                                               feed_forward_proj="gated-gelu", tie_word_embeddings=False),
                            t.T5ForConditionalGeneration),
        "t5_encoder": (lambda: t.T5Config(d_model=64, d_kv=16, d_ff=128, num_heads=4, num_layers=2, vocab_size=100),
                       t.T5EncoderModel),
        "mt5": (lambda: t.MT5Config(d_model=64, d_kv=16, d_ff=128, num_heads=4, num_layers=1, vocab_size=120),
                t.MT5ForConditionalGeneration),
        "whisper": (lambda: t.WhisperConfig(d_model=64, encoder_layers=2, decoder_layers=1, encoder_attention_heads=4,
                                            decoder_attention_heads=4, encoder_ffn_dim=128, decoder_ffn_dim=96,
                                            vocab_size=100, num_mel_bins=80, max_source_positions=30,
                                            max_target_positions=20, decoder_start_token_id=1, **_IDS),
                    t.WhisperForConditionalGeneration),
        "mamba": (lambda: t.MambaConfig(hidden_size=64, num_hidden_layers=2, vocab_size=100, state_size=16, expand=2,
                                        conv_kernel=4), t.MambaForCausalLM),
        "mamba2": (lambda: t.Mamba2Config(hidden_size=64, num_hidden_layers=2, vocab_size=100, state_size=16,
                                          n_groups=2, head_dim=16, num_heads=8, expand=2), t.Mamba2ForCausalLM),
        "bamba": (lambda: t.BambaConfig(hidden_size=64, num_hidden_layers=3, vocab_size=100, num_attention_heads=4,
                                        num_key_value_heads=2, intermediate_size=128, attn_layer_indices=[1],
                                        mamba_n_heads=8, mamba_d_head=16, mamba_n_groups=2, mamba_d_state=16,
                                        mamba_expand=2), t.BambaForCausalLM),
        "gemma3_text": (lambda: t.Gemma3TextConfig(hidden_size=64, num_hidden_layers=7, vocab_size=100,
                                                   num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                                                   intermediate_size=128), t.Gemma3ForCausalLM),
        "gemma4_text": (lambda: t.Gemma4TextConfig(hidden_size=64, num_hidden_layers=4, vocab_size=100,
                                                   num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                                                   global_head_dim=64, intermediate_size=128,
                                                   hidden_size_per_layer_input=16, vocab_size_per_layer_input=50,
                                                   layer_types=["sliding_attention", "full_attention"] * 2),
                        t.Gemma4ForCausalLM),
        "gemma4_text_moe": (lambda: t.Gemma4TextConfig(
            hidden_size=64, num_hidden_layers=4, vocab_size=100, num_attention_heads=4, num_key_value_heads=2,
            head_dim=32, global_head_dim=64, num_global_key_value_heads=1, attention_k_eq_v=True,
            intermediate_size=128, hidden_size_per_layer_input=0, num_kv_shared_layers=2, use_double_wide_mlp=True,
            enable_moe_block=True, num_experts=4, top_k_experts=2, moe_intermediate_size=32,
            layer_types=["sliding_attention", "full_attention"] * 2), t.Gemma4ForCausalLM),
        "olmoe": (lambda: t.OlmoeConfig(hidden_size=64, num_hidden_layers=2, vocab_size=100, num_attention_heads=4,
                                        num_key_value_heads=2, intermediate_size=32, num_experts=4,
                                        num_experts_per_tok=2), t.OlmoeForCausalLM),
        "deepseek_v2": (lambda: t.DeepseekV2Config(
            hidden_size=64, num_hidden_layers=3, vocab_size=100, num_attention_heads=4, num_key_value_heads=4,
            intermediate_size=128, moe_intermediate_size=32, n_routed_experts=4, n_shared_experts=2,
            num_experts_per_tok=2, first_k_dense_replace=1, q_lora_rank=24, kv_lora_rank=16, qk_nope_head_dim=16,
            qk_rope_head_dim=8, v_head_dim=16), t.DeepseekV2ForCausalLM),
        "deepseek_v2_lite": (lambda: t.DeepseekV2Config(
            hidden_size=64, num_hidden_layers=2, vocab_size=100, num_attention_heads=4, num_key_value_heads=4,
            intermediate_size=128, moe_intermediate_size=32, n_routed_experts=4, n_shared_experts=1,
            num_experts_per_tok=2, first_k_dense_replace=1, q_lora_rank=None, kv_lora_rank=16, qk_nope_head_dim=16,
            qk_rope_head_dim=8, v_head_dim=16), t.DeepseekV2ForCausalLM),
        "llava": (lambda: t.LlavaConfig(text_config=dict(llama, model_type="llama"),
                                        vision_config=dict(clip_vision, model_type="clip_vision_model")),
                  t.LlavaForConditionalGeneration),
        "llava_qwen2_siglip": (lambda: t.LlavaConfig(
            text_config=dict(llama, model_type="qwen2"), vision_config=dict(clip_vision, model_type="siglip_vision_model"),
            multimodal_projector_bias=False), t.LlavaForConditionalGeneration),
        "mllama": (lambda: t.MllamaConfig(
            text_config=dict(hidden_size=64, num_hidden_layers=4, vocab_size=100, num_attention_heads=4,
                             num_key_value_heads=2, intermediate_size=128, cross_attention_layers=[1, 3], **_IDS),
            vision_config=dict(hidden_size=48, intermediate_size=96, num_hidden_layers=2, num_global_layers=1,
                               attention_heads=4, image_size=32, patch_size=8, max_num_tiles=4, vision_output_dim=96,
                               intermediate_layers_indices=[0])), t.MllamaForConditionalGeneration),
        "qwen3_vl": (lambda: t.Qwen3VLConfig(
            text_config=dict(hidden_size=64, num_hidden_layers=2, vocab_size=100, num_attention_heads=4,
                             num_key_value_heads=2, intermediate_size=128, head_dim=16),
            vision_config=dict(depth=3, hidden_size=48, intermediate_size=96, num_heads=4, patch_size=8,
                               temporal_patch_size=2, spatial_merge_size=2, out_hidden_size=64,
                               num_position_embeddings=64, deepstack_visual_indexes=[0, 2])),
                     t.Qwen3VLForConditionalGeneration),
    }


FAMILIES = list(_family_configs())
FAMILY_OF = {"bert_mlm": "bert", "bert_seq": "bert", "bert_tok": "bert", "xlm_roberta_rerank": "xlm_roberta",
             "clip_text": "clip", "clip_vision": "clip", "clip_text_plain": "clip", "siglip_vision": "siglip",
             "t5_gated_untied": "t5", "t5_encoder": "t5", "mt5": "t5", "gemma4_text_moe": "gemma4_text",
             "deepseek_v2_lite": "deepseek_v2", "llava_qwen2_siglip": "llava"}


def _split_experts(shapes):
    """transformers' fused expert tensors -> the per-expert matrices the hub checkpoints hold."""
    out = {}
    for name, shape in shapes.items():
        m = re.fullmatch(r"(.*\.mlp\.experts)\.(gate_up_proj|down_proj)", name)
        if m is None:
            out[name] = shape
            continue
        E, rows, cols = shape
        for e in range(E):
            p = f"{m.group(1)}.{e}"
            if m.group(2) == "gate_up_proj":
                out[f"{p}.gate_proj.weight"] = (rows // 2, cols)
                out[f"{p}.up_proj.weight"] = (rows // 2, cols)
            else:
                out[f"{p}.down_proj.weight"] = (rows, cols)
    return out


def _oracle(key):
    """The transformers module's config.json and its checkpoint's names and shapes."""
    make, cls = _family_configs()[key]
    cfg = make()
    with torch.device("meta"):
        model = cls(cfg)
    shapes = {n: tuple(t.shape) for n, t in model.state_dict().items()}
    conf = json.loads(cfg.to_json_string())
    conf["architectures"] = [cls.__name__]
    tied = getattr(model, "_tied_weights_keys", None) or {}
    tied = tied if isinstance(tied, dict) else {k: None for k in tied}
    if not key.startswith("gemma4"):  # Gemma-4 checkpoints keep the fused expert tensors
        shapes = _split_experts(shapes)
    return conf, shapes, tied


def _write(directory, conf, shapes):
    directory.mkdir(parents=True, exist_ok=True)
    (directory / "config.json").write_text(json.dumps(conf))
    synthetic.write_headers(str(directory), shapes)
    return engine.Checkpoint.declared(str(directory))


@pytest.mark.parametrize("key", FAMILIES)
def test_composition_reads_every_tensor_of_the_transformers_module(tmp_path, key):
    conf, shapes, tied = _oracle(key)
    comp = catalog.compose(_write(tmp_path / "all", conf, shapes))
    assert comp.family == FAMILY_OF.get(key, key)
    assert comp.architecture == conf["architectures"][0]
    assert comp.architecture in catalog.architectures()
    # Every name and shape of the module, none added: the weights, plus the optional ones it holds.
    assert {**comp.weights, **{n: s for n, s in comp.optional.items() if n in shapes}} == shapes
    # A checkpoint saved without its optional weights (tied copies, as save_pretrained writes) fits.
    held = {n: s for n, s in shapes.items() if n not in comp.optional}
    assert catalog.compose(_write(tmp_path / "held", conf, held)).weights == held
    assert comp.parameters() == sum(torch.Size(s).numel() for s in held.values())
    assert comp.describe().startswith(comp.tree[0]) and len(comp.tree) >= 2
    # What is optional is a tied copy or a part the model may leave out.
    for name in comp.optional:
        assert name in tied or "pooler" in name, name


def test_bert_checkpoints_nest_the_encoder_and_keep_pretraining_heads(tmp_path):
    conf, shapes, _ = _oracle("bert")
    nested = {"bert." + n: s for n, s in shapes.items()}
    nested["cls.seq_relationship.weight"] = (2, 64)
    nested["bert.embeddings.position_ids"] = (1, 40)
    comp = catalog.compose(_write(tmp_path / "a", conf, nested))
    assert set(comp.weights) == {n for n in nested if not n.startswith("cls.") and not n.endswith("position_ids")}
    conf, shapes, _ = _oracle("bert_mlm")
    extra = dict(shapes, **{"cls.seq_relationship.weight": (2, 64), "bert.pooler.dense.weight": (64, 64)})
    assert catalog.compose(_write(tmp_path / "b", conf, extra)).weights.keys() == {
        n for n in shapes if n not in ("cls.predictions.decoder.weight", "cls.predictions.decoder.bias")}


@pytest.mark.parametrize("key", ["llava", "mllama"])
def test_vision_language_reads_the_hub_exports_layout(tmp_path, key):
    """The first hub exports name the text decoder `language_model.model.*`, its head
    `language_model.lm_head.weight`, and keep the vision tower and projector at the root."""
    conf, shapes, _ = _oracle(key)

    def legacy(n):
        if n == "lm_head.weight":
            return "language_model.lm_head.weight"
        if n.startswith("model.language_model."):
            return "language_model.model." + n[len("model.language_model."):]
        return n[len("model."):] if n.startswith("model.") else n

    old = {legacy(n): s for n, s in shapes.items()}
    comp = catalog.compose(_write(tmp_path, conf, old))
    assert {**comp.weights, **{n: s for n, s in comp.optional.items() if n in old}} == old


def test_gemma_trees_count_global_and_sliding_layers(tmp_path):
    conf, shapes, _ = _oracle("gemma3_text")
    comp = catalog.compose(_write(tmp_path / "a", conf, shapes))
    want = conf["layer_types"].count("full_attention")
    assert f"({want} global, {7 - want} sliding-window" in comp.tree[0]
    bad = dict(conf, layer_types=conf["layer_types"][:3])
    with pytest.raises(ValueError, match="config.json:layer_types"):
        catalog.compose(_write(tmp_path / "b", bad, shapes))
    conf, shapes, _ = _oracle("gemma4_text_moe")
    comp = catalog.compose(_write(tmp_path / "c", conf, shapes))
    assert "the last 2 reuse earlier layers' KV; MoE block" in comp.tree[0]
    assert "model.layers.1.self_attn.v_proj.weight" not in comp.weights  # global layers use keys as values
    assert comp.weights["model.layers.3.mlp.gate_proj.weight"] == (256, 64)  # double-wide shared-KV layer


@pytest.mark.parametrize("key", ["bert", "whisper", "mamba2", "clip", "deepseek_v2", "qwen3_vl"])
def test_refuses_missing_misshaped_and_unread_tensors(tmp_path, key):
    conf, shapes, _ = _oracle(key)
    comp = catalog.compose(_write(tmp_path / "ok", conf, shapes))
    name = sorted(comp.weights)[len(comp.weights) // 2]
    missing = {n: s for n, s in shapes.items() if n != name}
    with pytest.raises(ValueError, match=f"{re.escape(name)}: missing from the checkpoint"):
        catalog.compose(_write(tmp_path / "missing", conf, missing))
    misshaped = dict(shapes, **{name: tuple(d + 1 for d in shapes[name]) or (2,)})
    with pytest.raises(ValueError, match=f"{re.escape(name)}: shape"):
        catalog.compose(_write(tmp_path / "shape", conf, misshaped))
    extra = dict(shapes, **{"extra.weight": (4,)})
    with pytest.raises(ValueError, match="extra.weight: not read by the"):
        catalog.compose(_write(tmp_path / "extra", conf, extra))
    # Unchecked, the composition is the config's alone.
    assert catalog.compose(_write(tmp_path / "extra2", conf, extra), check=False).weights == comp.weights


def test_refuses_configs_without_a_composition_or_a_consistent_geometry(tmp_path):
    conf, shapes, _ = _oracle("t5")
    with pytest.raises(ValueError, match="config.json:d_kv"):
        catalog.compose(_write(tmp_path / "a", {k: v for k, v in conf.items() if k != "d_kv"}, shapes))
    with pytest.raises(ValueError, match="no catalog composition"):
        catalog.compose(_write(tmp_path / "b", dict(conf, architectures=["Qwen3ForCausalLM"]), shapes))
    conf, shapes, _ = _oracle("mamba2")
    with pytest.raises(ValueError, match="config.json:num_heads"):
        catalog.compose(_write(tmp_path / "c", dict(conf, num_heads=6), shapes))
    conf, shapes, _ = _oracle("bamba")
    with pytest.raises(ValueError, match="config.json:attn_layer_indices: layer 7 out of range"):
        catalog.compose(_write(tmp_path / "d", dict(conf, attn_layer_indices=[7]), shapes))
    conf, shapes, _ = _oracle("qwen3_vl")
    bad = dict(conf, vision_config=dict(conf["vision_config"], out_hidden_size=32))
    with pytest.raises(ValueError, match="config.json:vision_config.out_hidden_size"):
        catalog.compose(_write(tmp_path / "e", bad, shapes))
    conf, shapes, _ = _oracle("llava")
    bad = dict(conf, text_config=dict(conf["text_config"], model_type="gemma"))
    with pytest.raises(ValueError, match="config.json:text_config.model_type"):
        catalog.compose(_write(tmp_path / "f", bad, shapes))
    assert catalog.composes("WhisperForConditionalGeneration")
    assert not catalog.composes("LlamaForCausalLM")


def test_nested_configs_take_the_upstream_defaults(tmp_path):
    """Older exports keep only the sub-config values that differ from the class defaults: a LLaVA
    text config that names its vocabulary alone is a Llama-7B decoder."""
    conf = {"architectures": ["LlavaForConditionalGeneration"], "text_config": {"model_type": "llama",
            "vocab_size": 32064}, "vision_config": {"hidden_size": 1024, "image_size": 336, "intermediate_size": 4096,
            "model_type": "clip_vision_model", "num_attention_heads": 16, "num_hidden_layers": 24, "patch_size": 14}}
    comp = catalog.compose(_write(tmp_path, conf, {}), check=False)
    assert comp.weights["model.language_model.layers.31.mlp.gate_proj.weight"] == (11008, 4096)
    assert comp.weights["model.vision_tower.vision_model.embeddings.position_embedding.weight"] == (577, 1024)
    assert comp.weights["lm_head.weight"] == (32064, 4096)
    assert 7.0e9 < comp.parameters() < 7.1e9


@pytest.mark.parametrize("key", ["bert", "t5", "whisper", "mamba2", "gemma3_text", "clip", "llava", "olmoe"])
def test_registry_still_refuses_to_load_a_catalog_family(tmp_path, key):
    conf, shapes, _ = _oracle(key)
    ck = _write(tmp_path, conf, shapes)
    with pytest.raises(NotImplementedError, match="no model type is implemented"):
        engine.LoadOptions().parse(ck)


def test_every_catalog_architecture_is_a_registry_name():
    from furiosa_opt_engine import _native

    names = set(_native._architectures())
    assert set(catalog.architectures()) <= names


# ---- Diffusion: no diffusers in the image, so the oracle is the published parameter counts ----

SD_VAE = {"_class_name": "AutoencoderKL", "block_out_channels": [128, 256, 512, 512],
          "down_block_types": ["DownEncoderBlock2D"] * 4, "up_block_types": ["UpDecoderBlock2D"] * 4,
          "in_channels": 3, "out_channels": 3, "latent_channels": 4, "layers_per_block": 2, "norm_num_groups": 32}
FLUX_VAE = dict(SD_VAE, latent_channels=16, use_quant_conv=False, use_post_quant_conv=False)
FLUX_DEV = {"_class_name": "FluxTransformer2DModel", "attention_head_dim": 128, "guidance_embeds": True,
            "in_channels": 64, "joint_attention_dim": 4096, "num_attention_heads": 24, "num_layers": 19,
            "num_single_layers": 38, "patch_size": 1, "pooled_projection_dim": 768, "axes_dims_rope": [16, 56, 56]}
DIT_XL_2 = {"_class_name": "Transformer2DModel", "activation_fn": "gelu-approximate", "attention_bias": True,
            "attention_head_dim": 72, "in_channels": 4, "norm_type": "ada_norm_zero", "num_attention_heads": 16,
            "num_embeds_ada_norm": 1000, "num_layers": 28, "out_channels": 8, "patch_size": 2, "sample_size": 32}


def _compose_config(tmp_path, name, cfg, check=False):
    d = tmp_path / name
    d.mkdir(parents=True, exist_ok=True)
    (d / "config.json").write_text(json.dumps(cfg))
    return catalog.compose(engine.Checkpoint.declared(str(d)), check=check)


def test_diffusion_compositions_hold_the_published_parameter_counts(tmp_path):
    assert _compose_config(tmp_path, "sd_vae", SD_VAE).parameters() == 83_653_863  # Stable Diffusion's VAE
    assert _compose_config(tmp_path, "flux_vae", FLUX_VAE).parameters() == 83_819_683  # FLUX.1's VAE
    flux = _compose_config(tmp_path, "flux", FLUX_DEV)
    assert flux.parameters() == 11_901_408_320  # FLUX.1-dev's transformer
    assert flux.family == "flux" and "transformer_blocks.18.attn.norm_added_k.weight" in flux.weights
    schnell = _compose_config(tmp_path, "schnell", dict(FLUX_DEV, guidance_embeds=False))
    assert flux.parameters() - schnell.parameters() == 2 * 3072 + 256 * 3072 + 3072 * 3072
    # DiT-XL/2: 675,129,632 in the original code, which counts its fixed 256 x 1152 position table
    # and shares one timestep and class embedder; diffusers gives every block its own embedders.
    dit = _compose_config(tmp_path, "dit", DIT_XL_2)
    embedders = (256 * 1152 + 1152 + 1152 * 1152 + 1152) + 1001 * 1152
    assert dit.parameters() - 27 * embedders + 256 * 1152 == 675_129_632
    assert "pos_embed.pos_embed" in dit.ignored


def test_diffusion_refusals(tmp_path):
    with pytest.raises(ValueError, match="config.json:norm_type: ada_norm_single"):
        _compose_config(tmp_path, "a", dict(DIT_XL_2, norm_type="ada_norm_single"))
    with pytest.raises(ValueError, match="config.json:down_block_types: every block is DownEncoderBlock2D"):
        _compose_config(tmp_path, "b", dict(SD_VAE, down_block_types=["DownBlock2D"] * 4))
    with pytest.raises(ValueError, match="config.json:block_out_channels: 100 channels in groups of 32"):
        _compose_config(tmp_path, "c", dict(SD_VAE, block_out_channels=[128, 100, 512, 512]))
    with pytest.raises(ValueError, match="config.json:axes_dims_rope"):
        _compose_config(tmp_path, "d", dict(FLUX_DEV, axes_dims_rope=[16, 56, 48]))


def _tiny_flux_pipeline(root):
    """A FLUX pipeline folder of tiny geometry: model_index.json and four components, each with its
    config and a header-only safetensors file (text encoders from transformers' modules)."""
    t = transformers
    root.mkdir(parents=True, exist_ok=True)
    (root / "model_index.json").write_text(json.dumps({
        "_class_name": "FluxPipeline", "scheduler": ["diffusers", "FlowMatchEulerDiscreteScheduler"],
        "text_encoder": ["transformers", "CLIPTextModel"], "text_encoder_2": ["transformers", "T5EncoderModel"],
        "tokenizer": ["transformers", "CLIPTokenizer"], "transformer": ["diffusers", "FluxTransformer2DModel"],
        "vae": ["diffusers", "AutoencoderKL"]}))
    shapes = {}
    for name, cfg, cls in [("text_encoder", t.CLIPTextConfig(hidden_size=32, intermediate_size=64, num_hidden_layers=1,
                                                             num_attention_heads=2, vocab_size=50,
                                                             max_position_embeddings=16), t.CLIPTextModel),
                           ("text_encoder_2", t.T5Config(d_model=32, d_kv=8, d_ff=64, num_heads=4, num_layers=1,
                                                         vocab_size=50), t.T5EncoderModel)]:
        with torch.device("meta"):
            model = cls(cfg)
        conf = json.loads(cfg.to_json_string())
        conf["architectures"] = [cls.__name__]
        d = root / name
        d.mkdir()
        (d / "config.json").write_text(json.dumps(conf))
        held = {n: tuple(v.shape) for n, v in model.state_dict().items() if n != "encoder.embed_tokens.weight"}
        synthetic.write_headers(str(d), held)
        shapes.update({f"{name}.{n}": s for n, s in held.items()})
    for name, cfg in [("transformer", dict(FLUX_DEV, num_layers=1, num_single_layers=2, num_attention_heads=2,
                                           attention_head_dim=16, axes_dims_rope=[4, 6, 6], joint_attention_dim=32,
                                           pooled_projection_dim=32, in_channels=16)),
                      ("vae", dict(SD_VAE, block_out_channels=[32, 64], down_block_types=["DownEncoderBlock2D"] * 2,
                                   up_block_types=["UpDecoderBlock2D"] * 2, latent_channels=4, layers_per_block=1))]:
        d = root / name
        d.mkdir()
        (d / "config.json").write_text(json.dumps(cfg))
        comp = catalog.compose(engine.Checkpoint.declared(str(d)), check=False)
        synthetic.write_headers(str(d), comp.weights)
        shapes.update({f"{name}.{n}": s for n, s in comp.weights.items()})
    (root / "scheduler").mkdir()
    (root / "scheduler" / "scheduler_config.json").write_text(json.dumps({"_class_name": "FlowMatchEulerDiscreteScheduler"}))
    return shapes


def test_pipelines_compose_each_component_under_its_folder(tmp_path):
    shapes = _tiny_flux_pipeline(tmp_path / "flux")
    comp = catalog.compose(engine.Checkpoint.declared(str(tmp_path / "flux")))
    assert comp.family == "pipeline" and comp.architecture == "FluxPipeline"
    assert comp.weights == shapes
    assert {line.strip().split(":")[0] for line in comp.tree[1:] if line.startswith("  ") and not line.startswith("    ")} \
        == {"text_encoder", "text_encoder_2", "transformer", "vae"}
    assert "text_encoder_2.encoder.embed_tokens.weight" in comp.optional
    with pytest.raises(NotImplementedError, match="FluxPipeline"):
        engine.LoadOptions().parse(engine.Checkpoint.declared(str(tmp_path / "flux")))
    # A component whose tensor is missing is refused by its full name.
    (tmp_path / "flux" / "vae" / "model.safetensors").unlink()
    with pytest.raises(ValueError, match="vae.encoder.conv_in.weight: missing from the checkpoint"):
        catalog.compose(engine.Checkpoint.declared(str(tmp_path / "flux")))


def test_pipeline_components_without_a_composition_are_refused(tmp_path):
    shapes = _tiny_flux_pipeline(tmp_path / "p")
    assert shapes
    cfg = json.loads((tmp_path / "p" / "vae" / "config.json").read_text())
    (tmp_path / "p" / "vae" / "config.json").write_text(json.dumps(dict(cfg, _class_name="AutoencoderTiny")))
    with pytest.raises(ValueError, match="config.json:vae: AutoencoderTiny has no catalog composition"):
        catalog.compose(engine.Checkpoint.declared(str(tmp_path / "p")))
