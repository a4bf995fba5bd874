"""The registry and load options: every name once, lookups and refusals by kind and message, and
the choices a load makes from a config alone (no weight is read, no device opened)."""

import json
import os

import pytest

import furiosa_opt_engine as engine
from furiosa_opt_engine import _native
from furiosa_opt_models_b200.models import configs, synthetic


def test_lists_every_name_once():
    names = _native._architectures()
    assert len(names) == 670
    assert len(set(names)) == 670


def _ckpt(tmp_path, config):
    d = tmp_path / "ck"
    d.mkdir(parents=True, exist_ok=True)
    return engine.Checkpoint(str(d), config)


def test_selects_the_first_listed_architecture(tmp_path):
    unknown = "UnknownForCausalLM"
    with pytest.raises(ValueError, match="config.json:hidden_size"):
        engine.LoadOptions().parse(_ckpt(tmp_path, {"architectures": [unknown, "Qwen3ForCausalLM"]}))
    with pytest.raises(NotImplementedError, match="ApertusForCausalLM: no model type is implemented"):
        engine.LoadOptions().parse(_ckpt(tmp_path, {"architectures": [unknown, "ApertusForCausalLM", "Qwen3ForCausalLM"]}))
    with pytest.raises(NotImplementedError, match="FluxPipeline"):
        engine.LoadOptions().parse(_ckpt(tmp_path, {"architectures": [unknown], "_class_name": "FluxPipeline"}))
    with pytest.raises(ValueError, match="UnknownForCausalLM, UnknownModel: unknown architecture"):
        engine.LoadOptions().parse(_ckpt(tmp_path, {"architectures": [unknown, "UnknownModel"]}))
    with pytest.raises(ValueError, match="the config names no architecture"):
        engine.LoadOptions().parse(_ckpt(tmp_path, {}))


@pytest.mark.parametrize("name,size", [("qwen3-1.7b", "1.7B"), ("qwen3-8b", "8B"), ("llama-3.1-8b", "8B"),
                                       ("llama-3.3-70b", "70B"), ("tiny-qwen3", "custom")])
def test_parse_reads_the_config_alone(tmp_path, name, size):
    cfg = synthetic.hf_config(configs.get(name))
    sel = engine.LoadOptions().select(_ckpt(tmp_path, cfg))
    assert sel["size"] == size
    assert sel["precision"] == "bfloat16"


def test_option_refusals(tmp_path):
    ck = _ckpt(tmp_path, synthetic.hf_config(configs.get("qwen3-1.7b")))
    with pytest.raises(ValueError, match="chips: a model loads onto at least one chip"):
        engine.LoadOptions().chips(0)
    with pytest.raises(ValueError):
        engine.LoadOptions().kv_cache("nonsense")
    with pytest.raises(NotImplementedError, match="kv_cache: every implementation caches keys and values in BF16"):
        engine.LoadOptions().kv_cache("float16").parse(ck)
    with pytest.raises(NotImplementedError, match="layers: every implementation loads whole"):
        engine.LoadOptions().layers(range(0, 4)).parse(ck)
    with pytest.raises(ValueError):
        engine.LoadOptions().layers(range(0, 4, 2))
    with pytest.raises(ValueError, match="a quantization is fp8_per_tensor or fp8_per_channel"):
        engine.LoadOptions().quantization("int4")
    engine.LoadOptions().adapters().parse(ck)  # dense BF16 decoders take LoRA adapters
    moe = _ckpt(tmp_path / "moe", synthetic.hf_config(configs.get("tiny-qwen3-moe")))
    with pytest.raises(NotImplementedError, match="takes no adapter"):
        engine.LoadOptions().adapters().parse(moe)
    with pytest.raises(NotImplementedError, match="chips: a load runs on 1, 2, 4 or 8 chips"):
        engine.LoadOptions().chips(3).parse(ck)
    assert engine.LoadOptions().chips(8).select(ck)["chips"] == 8
    with pytest.raises(ValueError, match="unknown architecture"):
        engine.LoadOptions().architecture("NoSuchForCausalLM")
    with pytest.raises(NotImplementedError, match="no model type is implemented"):
        engine.LoadOptions().architecture("BloomForCausalLM")
    assert engine.LoadOptions().architecture("Qwen3ForCausalLM").batch_invariant().select(ck)["class"] == "qwen3.ForCausalLM"


def test_qwen3_refusals(tmp_path):
    base = synthetic.hf_config(configs.get("qwen3-1.7b"))
    with pytest.raises(NotImplementedError, match="use_sliding_window: Qwen3 attends the whole history"):
        engine.LoadOptions().parse(_ckpt(tmp_path, dict(base, use_sliding_window=True)))
    with pytest.raises(NotImplementedError, match="attention_bias"):
        engine.LoadOptions().parse(_ckpt(tmp_path, dict(base, attention_bias=True)))
    with pytest.raises(NotImplementedError, match="rope_scaling"):
        engine.LoadOptions().parse(_ckpt(tmp_path, dict(base, rope_scaling={"rope_type": "dynamic", "factor": 2.0})))


def test_classes_of_the_family(tmp_path):
    base = synthetic.hf_config(configs.get("qwen3-0.6b"))
    for arch, cls in [("Qwen3ForSequenceClassification", "qwen3.ForSequenceClassification"),
                      ("Qwen3Model", "qwen3.Model")]:
        assert engine.LoadOptions().select(_ckpt(tmp_path, dict(base, architectures=[arch])))["class"] == cls


def test_media_encoder_loads_alone(tmp_path):
    """Gemma 4 unified's media embedders are an Encoder a load of the encoder alone returns; the
    reference refuses the other combinations (vision_language/gemma4_unified.rs:25-33, the
    decoders' `reads(Part)`, models/vision_language/gemma4_unified.rs:127-164)."""
    ck = _ckpt(tmp_path, synthetic.gemma4_unified_config(3840, 3840, 1120, 640))
    sel = engine.LoadOptions().encoder().select(ck)
    assert sel["architecture"] == "Gemma4UnifiedForConditionalGeneration"
    assert sel["size"] == "12B"
    assert _native.LoadOptions().encoder().select(
        _ckpt(tmp_path / "small", synthetic.gemma4_unified_config()))["size"] == "custom"
    with pytest.raises(NotImplementedError, match="^encoder: a media encoder loads alone, so choose the encoder$"):
        engine.LoadOptions().parse(ck)
    with pytest.raises(NotImplementedError, match="^quantization: the media encoder's projections stay BF16$"):
        engine.LoadOptions().encoder().quantization("fp8_per_tensor").parse(ck)
    with pytest.raises(NotImplementedError, match="^chips: a media encoder runs on one chip$"):
        engine.LoadOptions().encoder().chips(2).parse(ck)
    qwen = _ckpt(tmp_path / "qwen", synthetic.hf_config(configs.get("qwen3-1.7b")))
    with pytest.raises(NotImplementedError, match="^encoder: a decoder holds no media encoder that loads alone$"):
        engine.LoadOptions().encoder().parse(qwen)


def test_media_encoder_refuses_odd_widths(tmp_path):
    odd = synthetic.gemma4_unified_config(text=250)
    with pytest.raises(NotImplementedError, match="hidden_size 250 is not a multiple of 64"):
        engine.LoadOptions().encoder().parse(_ckpt(tmp_path, odd))
    broken = synthetic.gemma4_unified_config()
    del broken["vision_config"]["mm_embed_dim"]
    with pytest.raises(ValueError, match="vision_config.mm_embed_dim"):
        engine.LoadOptions().encoder().parse(_ckpt(tmp_path / "b", broken))


@pytest.mark.parametrize("name,cls,size", [("mixtral-8x7b", "mixtral.ForCausalLM", "8x7B"),
                                           ("tiny-mixtral", "mixtral.ForCausalLM", "custom"),
                                           ("tiny-qwen3-moe", "qwen3_moe.ForCausalLM", "custom")])
def test_mixture_of_experts_families_load_from_the_config(tmp_path, name, cls, size):
    """Weightless loads of the mixture-of-experts families: the class, size and precision come from
    config.json alone."""
    sel = engine.LoadOptions().select(_ckpt(tmp_path, synthetic.hf_config(configs.get(name))))
    assert sel["class"] == cls and sel["size"] == size and sel["precision"] == "bfloat16"


def test_mixture_of_experts_refusals(tmp_path):
    base = synthetic.hf_config(configs.get("mixtral-8x7b"))
    with pytest.raises(NotImplementedError, match="sliding_window"):
        engine.LoadOptions().parse(_ckpt(tmp_path, dict(base, sliding_window=4096)))
    # Listed upstream but without an implementation: refused as not served, before any weight.
    for arch in ("OlmoeForCausalLM", "DeepseekV2ForCausalLM"):
        with pytest.raises(NotImplementedError, match=f"{arch}: no model type is implemented"):
            engine.LoadOptions().parse(_ckpt(tmp_path / arch, dict(base, architectures=[arch])))
