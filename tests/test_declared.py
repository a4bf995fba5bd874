"""Checkpoints too large to write, checked from headers alone (the reference's weightless
checkpoint tests, tests/common/mod.rs and qwen3_moe.rs:41): a header-only safetensors file
declares every tensor of the full-size geometry, `Checkpoint.declared` maps the names without
data, and the registry selects the class, size and chip split from it."""

import pytest

import furiosa_opt_engine as engine
from furiosa_opt_models_b200.models import configs, synthetic


@pytest.mark.parametrize("name", ["tiny-qwen3", "tiny-qwen3-moe", "tiny-mixtral"])
def test_shapes_match_the_written_weights(name):
    cfg = configs.get(name)
    assert synthetic.hf_shapes(cfg) == {k: tuple(v.shape) for k, v in synthetic.hf_weights(cfg).items()}


@pytest.mark.parametrize(("name", "cls", "size"), [
    ("qwen3-30b-a3b", "qwen3_moe.ForCausalLM", "30B-A3B"),
    ("mixtral-8x7b", "mixtral.ForCausalLM", "8x7B"),
    ("llama-3.3-70b", "llama.ForCausalLM", "70B"),
    ("llama-3.1-8b", "llama.ForCausalLM", "8B"),
    ("qwen3-8b", "qwen3.ForCausalLM", "8B"),
    ("qwen3-1.7b", "qwen3.ForCausalLM", "1.7B"),
])
def test_full_size_checkpoints_select_from_headers(tmp_path, name, cls, size):
    shapes = synthetic.write_declared(str(tmp_path), name)
    ck = engine.Checkpoint.declared(str(tmp_path))
    assert sorted(ck.names()) == sorted(shapes)
    engine.LoadOptions().parse(ck)
    for chips in (1, 2, 4, 8):
        sel = engine.LoadOptions().chips(chips).select(ck)
        assert (sel["class"], sel["size"], sel["chips"]) == (cls, size, chips)


@pytest.mark.parametrize(("name", "size", "precision"), [
    ("llama-3.1-8b-fp8", "8B", "float8_e4m3fn"),
    ("qwen3-8b-fp8", "8B", "float8_e4m3fn"),
    ("llama-3.3-70b-nvfp4", "70B", "uint8"),
    ("mistral-nemo-12b-fp8", "12B", "float8_e4m3fn"),
])
def test_quantized_full_size_checkpoints_select_their_format(tmp_path, name, size, precision):
    """The BASELINE-shaped quantized checkpoints (block-FP8 8B, NVFP4 70B), declared in their
    published formats, select the quantized line at every chip count."""
    shapes = synthetic.write_declared(str(tmp_path), name)
    ck = engine.Checkpoint.declared(str(tmp_path))
    assert sorted(ck.names()) == sorted(shapes)
    for chips in (1, 8):
        sel = engine.LoadOptions().chips(chips).select(ck)
        assert (sel["size"], sel["precision"], sel["chips"]) == (size, precision, chips)


def test_mixtral_refusals_name_the_option(tmp_path):
    """A sliding window or router noise is refused by name, before any weight is read."""
    import json
    import os

    synthetic.write_declared(str(tmp_path), "mixtral-8x7b")
    path = os.path.join(str(tmp_path), "config.json")
    base = json.load(open(path))
    for key, value in (("sliding_window", 4096), ("router_jitter_noise", 0.01)):
        with open(path, "w") as f:
            json.dump(dict(base, **{key: value}), f)
        with pytest.raises(NotImplementedError, match=key):
            engine.LoadOptions().select(engine.Checkpoint.declared(str(tmp_path)))
