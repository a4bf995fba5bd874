"""What a call returns besides greedy tokens (decoder.Output): a base model's final-normed hidden
rows (`Qwen3Model`, also saved with root-level names as sentence-embedding checkpoints are) and a
sequence classifier's FP32 scores with the label columns first (`Qwen3ForSequenceClassification`),
against the dense forward of the same weights. Neither reads a vocabulary head, so an untied
checkpoint without `lm_head.weight` loads."""

import json
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _write(directory, cfg, arch, tensors):
    from safetensors.torch import save_file

    from furiosa_opt_models_b200.models import synthetic

    os.makedirs(directory, exist_ok=True)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(dict(synthetic.hf_config(cfg), architectures=[arch]), f)
    save_file(tensors, os.path.join(directory, "model.safetensors"))


def _call(directory, prompt, keep_all=True):
    import furiosa_opt_engine as engine
    from furiosa_opt_engine import decoder as dec

    device = engine.Device(engine.Placement([0], range(8)))
    model = engine.LoadOptions().load(engine.Checkpoint(directory), device)
    cache = dec.Cache(model.cache, 8)
    toks = engine.HostTensor.from_dlpack(torch.tensor(prompt, dtype=torch.int32)).to_hbm(device)
    out = model.forward([dec.Request([list(range(8))], 0, toks, dec.Keep.ALL if keep_all else dec.Keep.LAST)], cache)
    return model, torch.from_numpy(out.to_host().numpy()).float()


@pytest.mark.parametrize("names", ["model.", "root"])
def test_base_model_returns_final_normed_hidden_rows(tmp_path, names):
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-qwen3", tied=False)
    hf = synthetic.hf_weights(cfg, seed=21, std=0.05)
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    tensors = {k: v for k, v in hf.items() if k != "lm_head.weight"}
    if names == "root":
        tensors = {k.removeprefix("model."): v for k, v in tensors.items()}
    _write(str(tmp_path / "m"), cfg, "Qwen3Model", tensors)
    prompt = torch.randint(0, cfg["vocab"], (21,), generator=torch.Generator().manual_seed(3)).tolist()
    model, got = _call(str(tmp_path / "m"), prompt)
    assert model.output == dec.Output.HIDDEN
    want = dense.forward(w, cfg, torch.tensor(prompt), head=False)
    assert got.shape == want.shape
    err = (got - want).abs().max().item()
    assert err <= 0.03 * max(1.0, want.abs().max().item()), err
    cos = torch.nn.functional.cosine_similarity(got, want, dim=-1)
    assert cos.min().item() > 0.999


def test_sequence_classifier_returns_label_scores(tmp_path):
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-qwen3", tied=False)
    hf = synthetic.hf_weights(cfg, seed=22, std=0.05)
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    labels = 3
    score = (torch.randn(labels, cfg["hidden"], generator=torch.Generator().manual_seed(5)) * 0.05).bfloat16()
    tensors = {k: v for k, v in hf.items() if k != "lm_head.weight"}
    tensors["score.weight"] = score
    _write(str(tmp_path / "c"), cfg, "Qwen3ForSequenceClassification", tensors)
    prompt = torch.randint(0, cfg["vocab"], (17,), generator=torch.Generator().manual_seed(4)).tolist()
    model, got = _call(str(tmp_path / "c"), prompt, keep_all=False)
    assert model.output == dec.Output.SCORES
    assert got.shape == (1, 256)
    h = dense.forward(w, cfg, torch.tensor(prompt), head=False)[-1:]
    want = h @ score.float().T
    assert torch.allclose(got[:, :labels], want, atol=2e-2, rtol=2e-2), (got[:, :labels], want)
    assert torch.count_nonzero(got[:, labels:]) == 0
