"""Checkpoints: safetensors files mapped by name (index or directory), a tensor held by two
files refused, host copies, pipelines' component names, against the safetensors oracle."""

import json
import os

import pytest
import torch
from safetensors.torch import save_file

import furiosa_opt_engine as engine
from furiosa_opt_models_b200.models import synthetic


def test_maps_index_shards(tmp_path):
    w = synthetic.write(str(tmp_path / "m"), "tiny-qwen3", shards=3)
    ck = engine.Checkpoint(str(tmp_path / "m"))
    assert sorted(ck.names()) == sorted(w)
    assert ck.config["architectures"] == ["Qwen3ForCausalLM"]
    assert ck.read().names() == ck.names()


def test_refuses_a_tensor_in_two_files(tmp_path):
    d = tmp_path / "dup"
    d.mkdir()
    save_file({"a": torch.zeros(2)}, str(d / "one.safetensors"))
    save_file({"a": torch.ones(2)}, str(d / "two.safetensors"))
    (d / "config.json").write_text("{}")
    with pytest.raises(ValueError, match="a: held by two files"):
        engine.Checkpoint(str(d))


def test_config_argument_replaces_the_directory_config(tmp_path):
    synthetic.write(str(tmp_path / "m"), "tiny-qwen3")
    ck = engine.Checkpoint(str(tmp_path / "m"), {"architectures": ["LlamaForCausalLM"]})
    assert ck.config == {"architectures": ["LlamaForCausalLM"]}


def test_pipeline_components_are_named_by_folder(tmp_path):
    d = tmp_path / "pipe"
    (d / "vae" / "decoder").mkdir(parents=True)
    (d / "model_index.json").write_text(json.dumps({"_class_name": "FluxPipeline"}))
    save_file({"w": torch.zeros(2)}, str(d / "vae" / "decoder" / "x.safetensors"))
    (d / "vae" / "config.json").write_text(json.dumps({"k": 1}))
    ck = engine.Checkpoint(str(d))
    assert ck.names() == ["vae.decoder.w"]
    assert ck.config["vae"] == {"k": 1}
    with pytest.raises(NotImplementedError, match="FluxPipeline: no model type is implemented"):
        engine.LoadOptions().parse(ck)


def test_missing_directory_is_an_os_error(tmp_path):
    with pytest.raises(OSError):
        engine.Checkpoint(str(tmp_path / "none"))
