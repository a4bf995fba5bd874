"""Catalog compositions (BERT, T5/mT5, Whisper, Mamba-2, Gemma-3 text): built from config.json
alone and checked strictly against checkpoint headers. The oracle of every name and shape is the
transformers module of the same config, built on the meta device (no values); the checkpoints hold
only safetensors headers (`Checkpoint.declared`)."""

import json

import pytest

import furiosa_opt_engine as engine
from furiosa_opt_models_b200.models import catalog, synthetic

transformers = pytest.importorskip("transformers")
torch = pytest.importorskip("torch")


def _family_configs():
    t = transformers
    return {
        "bert": (t.BertConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, intermediate_size=128,
                              vocab_size=100, max_position_embeddings=40), t.BertModel),
        "t5": (t.T5Config(d_model=64, d_kv=16, d_ff=128, num_heads=4, num_layers=2, num_decoder_layers=3,
                          vocab_size=100, feed_forward_proj="relu"), t.T5ForConditionalGeneration),
        "t5_gated_untied": (t.T5Config(d_model=64, d_kv=8, d_ff=96, num_heads=6, num_layers=1, vocab_size=100,
                                       feed_forward_proj="gated-gelu", tie_word_embeddings=False),
                            t.T5ForConditionalGeneration),
        "mt5": (t.MT5Config(d_model=64, d_kv=16, d_ff=128, num_heads=4, num_layers=1, vocab_size=120),
                t.MT5ForConditionalGeneration),
        "whisper": (t.WhisperConfig(d_model=64, encoder_layers=2, decoder_layers=1, encoder_attention_heads=4,
                                    decoder_attention_heads=4, encoder_ffn_dim=128, decoder_ffn_dim=96,
                                    vocab_size=100, num_mel_bins=80, max_source_positions=30,
                                    max_target_positions=20, pad_token_id=0, bos_token_id=1, eos_token_id=2,
                                    decoder_start_token_id=1), t.WhisperForConditionalGeneration),
        "mamba2": (t.Mamba2Config(hidden_size=64, num_hidden_layers=2, vocab_size=100, state_size=16, n_groups=2,
                                  head_dim=16, num_heads=8, expand=2), t.Mamba2ForCausalLM),
        "gemma3_text": (t.Gemma3TextConfig(hidden_size=64, num_hidden_layers=7, vocab_size=100,
                                           num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                                           intermediate_size=128), t.Gemma3ForCausalLM),
    }


FAMILIES = list(_family_configs())


def _oracle(key):
    """The transformers module's config.json and its state dict's names and shapes."""
    cfg, cls = _family_configs()[key]
    with torch.device("meta"):
        model = cls(cfg)
    shapes = {n: tuple(t.shape) for n, t in model.state_dict().items()}
    conf = json.loads(cfg.to_json_string())
    conf["architectures"] = [cls.__name__]
    tied = getattr(model, "_tied_weights_keys", None) or {}
    tied = tied if isinstance(tied, dict) else {k: None for k in tied}
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
    assert comp.family == key.split("_gated")[0].replace("mt5", "t5")
    assert comp.architecture == conf["architectures"][0]
    # Every name and shape of the module, none added: the weights, plus the tied copies it holds.
    assert {**comp.weights, **comp.aliases} == shapes
    assert set(comp.aliases) <= set(tied)
    # A checkpoint saved without its tied copies (as save_pretrained writes) fits as well.
    held = {n: s for n, s in shapes.items() if n not in comp.aliases}
    assert catalog.compose(_write(tmp_path / "untied", conf, held)).weights == held
    assert comp.parameters() == sum(torch.Size(s).numel() for s in held.values())
    assert comp.describe().startswith(comp.tree[0]) and len(comp.tree) >= 2


def test_bert_checkpoints_nest_the_encoder_under_bert(tmp_path):
    conf, shapes, _ = _oracle("bert")
    nested = {"bert." + n: s for n, s in shapes.items()}
    comp = catalog.compose(_write(tmp_path, conf, nested))
    assert set(comp.weights) == set(nested)


def test_gemma3_tree_counts_global_and_sliding_layers(tmp_path):
    conf, shapes, _ = _oracle("gemma3_text")
    comp = catalog.compose(_write(tmp_path / "a", conf, shapes))
    want = conf["layer_types"].count("full_attention")
    assert f"({want} global, {7 - want} sliding-window" in comp.tree[0]
    bad = dict(conf, layer_types=conf["layer_types"][:3])
    with pytest.raises(ValueError, match="config.json:layer_types"):
        catalog.compose(_write(tmp_path / "b", bad, shapes))


@pytest.mark.parametrize("key", ["bert", "whisper", "mamba2"])
def test_refuses_missing_misshaped_and_unread_tensors(tmp_path, key):
    conf, shapes, _ = _oracle(key)
    comp = catalog.compose(_write(tmp_path / "ok", conf, shapes))
    name = sorted(comp.weights)[len(comp.weights) // 2]
    missing = {n: s for n, s in shapes.items() if n != name}
    with pytest.raises(ValueError, match=f"{name}: missing from the checkpoint"):
        catalog.compose(_write(tmp_path / "missing", conf, missing))
    misshaped = dict(shapes, **{name: tuple(d + 1 for d in shapes[name])})
    with pytest.raises(ValueError, match=f"{name}: shape"):
        catalog.compose(_write(tmp_path / "shape", conf, misshaped))
    extra = dict(shapes, **{"extra.weight": (4,)})
    with pytest.raises(ValueError, match="extra.weight: not read by the"):
        catalog.compose(_write(tmp_path / "extra", conf, extra))
    # Unchecked, the composition is the config's alone.
    assert catalog.compose(_write(tmp_path / "extra2", conf, extra), check=False).weights == comp.weights


def test_refuses_configs_without_a_composition_or_a_geometry_key(tmp_path):
    conf, shapes, _ = _oracle("t5")
    with pytest.raises(ValueError, match="config.json:d_kv"):
        catalog.compose(_write(tmp_path / "a", {k: v for k, v in conf.items() if k != "d_kv"}, shapes))
    with pytest.raises(ValueError, match="no catalog composition"):
        catalog.compose(_write(tmp_path / "b", dict(conf, architectures=["Qwen3ForCausalLM"]), shapes))
    conf, shapes, _ = _oracle("mamba2")
    with pytest.raises(ValueError, match="config.json:num_heads"):
        catalog.compose(_write(tmp_path / "c", dict(conf, num_heads=6), shapes))
    assert catalog.composes("WhisperForConditionalGeneration")
    assert not catalog.composes("LlamaForCausalLM")


@pytest.mark.parametrize("key", ["bert", "t5", "whisper", "mamba2", "gemma3_text"])
def test_registry_still_refuses_to_load_a_catalog_family(tmp_path, key):
    conf, shapes, _ = _oracle(key)
    ck = _write(tmp_path, conf, shapes)
    with pytest.raises(NotImplementedError, match="no model type is implemented"):
        engine.LoadOptions().parse(ck)
