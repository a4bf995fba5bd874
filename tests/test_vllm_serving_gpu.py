"""vLLM through the plugin: vLLM's own LLM (scheduler, sampling parameters, request handling) on a
synthetic Qwen3 checkpoint, every forward pass in the engine; the greedy continuations agree with
the dense forward of the checkpoint's weights, and a sampled request is refused."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, "tests", "workers", "vllm_generate.py")


def test_vllm_generates_through_the_engine(tmp_path):
    pytest.importorskip("vllm")
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-qwen3")
    hf = synthetic.write(str(tmp_path / "m"), cfg, seed=11, std=0.05)
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    gen = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen).tolist() for n in (5, 17, 40)]
    out = str(tmp_path / "out.json")
    env = dict(os.environ, VLLM_PLUGINS="furiosa", VLLM_ENABLE_V1_MULTIPROCESSING="0",
               PYTHONPATH=os.pathsep.join([ROOT, os.path.join(ROOT, "integrations", "furiosa-opt-vllm")]))
    subprocess.run(["timeout", "-k", "30", "600", sys.executable, WORKER, str(tmp_path / "m"), out,
                    json.dumps(prompts)], check=True, env=env, cwd=ROOT)
    with open(out) as f:
        tokens = json.load(f)
    assert [len(t) for t in tokens] == [8, 8, 8]
    for p, toks in zip(prompts, tokens):
        seq = torch.tensor(p, dtype=torch.int32)
        for t in toks:
            logits = dense.forward(w, cfg, seq)[-1]
            assert logits[t] >= logits.max() - 1e-2 * max(1.0, abs(logits.max().item()))
            seq = torch.cat([seq, torch.tensor([t], dtype=torch.int32)])
    with open(out + ".refused") as f:
        assert json.load(f) is True


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_vllm_tensor_parallel_matches_the_dense_forward(tmp_path):
    """The parallelism contract through vLLM: the same checkpoint served at tensor_parallel_size 2
    (vLLM's multiprocess executor, one engine rank a worker) gives greedy tokens that are the dense
    forward's argmax at every step (within BF16 near-ties), as at TP=1."""
    pytest.importorskip("vllm")
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-qwen3-tp")
    hf = synthetic.write(str(tmp_path / "m"), cfg, seed=13, std=0.05)
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    gen = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen).tolist() for n in (5, 30)]
    env = dict(os.environ, VLLM_PLUGINS="furiosa", NCCL_NVLS_ENABLE="0",
               PYTHONPATH=os.pathsep.join([ROOT, os.path.join(ROOT, "integrations", "furiosa-opt-vllm")]))
    runs = {}
    for tp in (1, 2):
        out = str(tmp_path / f"tp{tp}.json")
        subprocess.run(["timeout", "-k", "30", "600", sys.executable, WORKER, str(tmp_path / "m"), out,
                        json.dumps(prompts), str(tp)], check=True, env=env, cwd=ROOT)
        with open(out) as f:
            runs[tp] = json.load(f)
    for tp, tokens in runs.items():
        for p, toks in zip(prompts, tokens):
            seq = torch.tensor(p, dtype=torch.int32)
            for t in toks:
                logits = dense.forward(w, cfg, seq)[-1]
                assert logits[t] >= logits.max() - 1e-2 * max(1.0, abs(logits.max().item())), tp
                seq = torch.cat([seq, torch.tensor([t], dtype=torch.int32)])


def test_vllm_sleep_mode_frees_and_restores(tmp_path):
    """vLLM's sleep mode through the plugin: level 1 keeps the host copy, level 2 reads the files,
    reload_weights loads them again; the continuations are the same each time, and sleeping
    returns the weights' and cache's device memory."""
    pytest.importorskip("vllm")
    from furiosa_opt_models_b200.models import configs, synthetic

    cfg = configs.get("tiny-qwen3")
    synthetic.write(str(tmp_path / "m"), cfg, seed=12, std=0.05)
    gen = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen).tolist() for n in (6, 21)]
    out = str(tmp_path / "sleep.json")
    env = dict(os.environ, VLLM_PLUGINS="furiosa", VLLM_ENABLE_V1_MULTIPROCESSING="0",
               PYTHONPATH=os.pathsep.join([ROOT, os.path.join(ROOT, "integrations", "furiosa-opt-vllm")]))
    subprocess.run(["timeout", "-k", "30", "600", sys.executable, os.path.join(ROOT, "tests", "workers", "vllm_sleep.py"),
                    str(tmp_path / "m"), out, json.dumps(prompts)], check=True, env=env, cwd=ROOT)
    with open(out) as f:
        r = json.load(f)
    assert r["before"] == r["level1"] == r["level2"] == r["reloaded"]
    assert r["freed_level1"] > 0


def test_vllm_lora_adapters(tmp_path):
    """Two PEFT LoRA adapters and none, in one vLLM batch: each continuation agrees with the dense
    forward of its merged weights."""
    pytest.importorskip("vllm")
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-qwen3")
    hf = synthetic.write(str(tmp_path / "m"), cfg, seed=13, std=0.05)
    base = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    paths, merged = [], []
    for i, (r, alpha) in enumerate([(8, 16.0), (16, 8.0)]):
        d = str(tmp_path / f"lora{i}")
        lora = synthetic.write_lora(d, cfg, r=r, alpha=alpha, seed=i + 1)
        paths.append(d)
        merged.append(synthetic.merge_lora(base, cfg, lora, r, alpha))
    prompt = torch.randint(0, cfg["vocab"], (11,), generator=torch.Generator().manual_seed(6)).tolist()
    out = str(tmp_path / "lora.json")
    env = dict(os.environ, VLLM_PLUGINS="furiosa", VLLM_ENABLE_V1_MULTIPROCESSING="0",
               PYTHONPATH=os.pathsep.join([ROOT, os.path.join(ROOT, "integrations", "furiosa-opt-vllm")]))
    subprocess.run(["timeout", "-k", "30", "600", sys.executable, os.path.join(ROOT, "tests", "workers", "vllm_lora.py"),
                    str(tmp_path / "m"), out, json.dumps(prompt), json.dumps(paths)], check=True, env=env, cwd=ROOT)
    with open(out) as f:
        tokens = json.load(f)
    for toks, w in zip(tokens, merged + [base]):
        seq = torch.tensor(prompt, dtype=torch.int32)
        for t in toks:
            logits = dense.forward(w, cfg, seq)[-1]
            assert logits[t] >= logits.max() - 1e-2 * max(1.0, abs(logits.max().item()))
            seq = torch.cat([seq, torch.tensor([t], dtype=torch.int32)])
    assert tokens[0] != tokens[2] or tokens[1] != tokens[2]


def test_vllm_ngram_speculation_is_exact(tmp_path):
    """n-gram speculative decoding through the plugin: drafts verified greedily by the engine give
    the same continuations as the dense forward of the checkpoint, and vLLM proposed drafts."""
    pytest.importorskip("vllm")
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-qwen3")
    hf = synthetic.write(str(tmp_path / "m"), cfg, seed=13, std=0.05)
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    gen = torch.Generator().manual_seed(6)
    # Repeating prompts, so prompt lookup finds n-grams to draft from.
    prompts = [[int(x) for x in torch.randint(0, cfg["vocab"], (4,), generator=gen)] * 6,
               torch.randint(0, cfg["vocab"], (19,), generator=gen).tolist()]
    out = str(tmp_path / "spec.json")
    env = dict(os.environ, VLLM_PLUGINS="furiosa", VLLM_ENABLE_V1_MULTIPROCESSING="0",
               PYTHONPATH=os.pathsep.join([ROOT, os.path.join(ROOT, "integrations", "furiosa-opt-vllm")]))
    subprocess.run(["timeout", "-k", "30", "600", sys.executable,
                    os.path.join(ROOT, "tests", "workers", "vllm_speculate.py"), str(tmp_path / "m"), out,
                    json.dumps(prompts)], check=True, env=env, cwd=ROOT)
    with open(out) as f:
        got = json.load(f)
    assert [len(t) for t in got["tokens"]] == [24, 24]
    for p, toks in zip(prompts, got["tokens"]):
        seq = torch.tensor(p, dtype=torch.int32)
        for t in toks:
            logits = dense.forward(w, cfg, seq)[-1]
            assert logits[t] >= logits.max() - 1e-2 * max(1.0, abs(logits.max().item()))
            seq = torch.cat([seq, torch.tensor([t], dtype=torch.int32)])
    drafts = got["counters"].get("vllm:spec_decode_num_draft_tokens")
    if drafts is not None:
        assert drafts > 0


def test_vllm_draft_model_speculation_is_exact(tmp_path):
    """Draft-model speculative decoding through the plugin: a smaller decoder of the same vocabulary
    (one layer, other weights) drafts beside the target; the target's greedy verification keeps the
    continuations equal to the dense forward of the target's weights."""
    pytest.importorskip("vllm")
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-qwen3")
    hf = synthetic.write(str(tmp_path / "m"), cfg, seed=13, std=0.05)
    synthetic.write(str(tmp_path / "d"), configs.get("tiny-qwen3", layers=1), seed=14, std=0.05)
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    gen = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen).tolist() for n in (9, 23)]
    out = str(tmp_path / "draft.json")
    env = dict(os.environ, VLLM_PLUGINS="furiosa", VLLM_ENABLE_V1_MULTIPROCESSING="0",
               PYTHONPATH=os.pathsep.join([ROOT, os.path.join(ROOT, "integrations", "furiosa-opt-vllm")]))
    subprocess.run(["timeout", "-k", "30", "600", sys.executable,
                    os.path.join(ROOT, "tests", "workers", "vllm_speculate.py"), str(tmp_path / "m"), out,
                    json.dumps(prompts), str(tmp_path / "d")], check=True, env=env, cwd=ROOT)
    with open(out) as f:
        got = json.load(f)
    assert [len(t) for t in got["tokens"]] == [24, 24]
    for p, toks in zip(prompts, got["tokens"]):
        seq = torch.tensor(p, dtype=torch.int32)
        for t in toks:
            logits = dense.forward(w, cfg, seq)[-1]
            assert logits[t] >= logits.max() - 1e-2 * max(1.0, abs(logits.max().item()))
            seq = torch.cat([seq, torch.tensor([t], dtype=torch.int32)])


def test_vllm_kv_offload_stores_and_loads_engine_pages(tmp_path):
    """KV offloading through the engine's connector: a prompt's pages go to host memory, other
    prompts evict them from the GPU, and the repeated prompt loads them back; its continuation is
    the same and the dense forward's."""
    pytest.importorskip("vllm")
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-qwen3")
    hf = synthetic.write(str(tmp_path / "m"), cfg, seed=15, std=0.05)
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    gen = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, cfg["vocab"], (256,), generator=gen).tolist() for _ in range(4)]
    out = str(tmp_path / "offload.json")
    env = dict(os.environ, VLLM_PLUGINS="furiosa", VLLM_ENABLE_V1_MULTIPROCESSING="0",
               PYTHONPATH=os.pathsep.join([ROOT, os.path.join(ROOT, "integrations", "furiosa-opt-vllm")]))
    subprocess.run(["timeout", "-k", "30", "600", sys.executable,
                    os.path.join(ROOT, "tests", "workers", "vllm_offload.py"), str(tmp_path / "m"), out,
                    json.dumps(prompts)], check=True, env=env, cwd=ROOT)
    with open(out) as f:
        got = json.load(f)
    assert got["first"] == got["again"], got
    assert got["stats"]["stored_blocks"] > 0 and got["stats"]["loaded_blocks"] > 0, got["stats"]
    seq = torch.tensor(prompts[0], dtype=torch.int32)
    for t in got["first"]:
        logits = dense.forward(w, cfg, seq)[-1]
        assert logits[t] >= logits.max() - 1e-2 * max(1.0, abs(logits.max().item()))
        seq = torch.cat([seq, torch.tensor([t], dtype=torch.int32)])


@pytest.mark.parametrize("mode", ["embed", "classify"])
def test_vllm_pooling_through_the_engine(tmp_path, mode):
    """vLLM's pooling runner through the plugin: `embed` on a causal checkpoint served as its base
    model (the normalized final hidden row of each prompt), `classify` on a sequence classifier
    (softmax of its label scores), against the dense forward."""
    pytest.importorskip("vllm")
    from safetensors.torch import save_file

    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-qwen3")
    d = tmp_path / "m"
    hf = synthetic.write(str(d), cfg, seed=14, std=0.05)
    synthetic.write_tokenizer(str(d), cfg["vocab"])  # vLLM's pooling front end opens one
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    score = None
    if mode == "classify":
        score = (torch.randn(3, cfg["hidden"], generator=torch.Generator().manual_seed(8)) * 0.05).bfloat16()
        save_file(dict(hf, **{"score.weight": score}), str(d / "model.safetensors"))
        conf = json.load(open(d / "config.json"))
        conf.update(architectures=["Qwen3ForSequenceClassification"], id2label={"0": "a", "1": "b", "2": "c"},
                    label2id={"a": 0, "b": 1, "c": 2})
        json.dump(conf, open(d / "config.json", "w"))
    gen = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen).tolist() for n in (7, 30)]
    out = str(tmp_path / "pool.json")
    env = dict(os.environ, VLLM_PLUGINS="furiosa", VLLM_ENABLE_V1_MULTIPROCESSING="0",
               PYTHONPATH=os.pathsep.join([ROOT, os.path.join(ROOT, "integrations", "furiosa-opt-vllm")]))
    subprocess.run(["timeout", "-k", "30", "600", sys.executable, os.path.join(ROOT, "tests", "workers", "vllm_pool.py"),
                    mode, str(d), out, json.dumps(prompts)], check=True, env=env, cwd=ROOT)
    with open(out) as f:
        got = json.load(f)
    for p, g in zip(prompts, got):
        h = dense.forward(w, cfg, torch.tensor(p), head=False)[-1]
        if mode == "embed":
            want = torch.nn.functional.normalize(h, dim=-1)
        else:
            want = torch.softmax(h @ score.float().T, -1)
        g = torch.tensor(g)
        assert g.shape == want.shape
        assert torch.allclose(g, want, atol=2e-2), (g, want)
