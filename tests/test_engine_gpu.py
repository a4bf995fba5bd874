"""The engine end to end on a GPU: a synthetic tiny Qwen3 decoder's paged prefill and greedy
decode against the dense FP32 PyTorch forward of the same weights."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _build(name="tiny-qwen3", **over):
    import furiosa_opt_engine as engine
    from furiosa_opt_models_b200.models import configs

    cfg = configs.get(name, **over)
    device = engine.Device(engine.Placement([0], range(8)))
    model = engine._native._synthetic_decoder(device, cfg, seed=7, std=0.05)
    return engine, cfg, device, model


def _weights(model):
    import dataclasses

    from furiosa_opt_models_b200.utils import devmem

    out = {}
    for k, v in devmem.weights(model).items():
        if isinstance(v, torch.Tensor):
            out[k] = v.float().cpu()
        else:
            out[k] = dataclasses.replace(v, codes=v.codes.cpu(), scales=v.scales.cpu())
    return out


@pytest.mark.parametrize("graphs", [True, False])
def test_prefill_then_greedy_decode_matches_dense(graphs):
    engine, cfg, device, model = _build()
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import dense

    model.set_graphs(graphs)
    w = _weights(model)
    lengths = [7, 16, 33, 64]
    gen = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen, dtype=torch.int32) for n in lengths]
    cache = dec.Cache(model.cache, 64)
    alloc = serving.BlockAllocator(64)
    seqs = [serving.Sequence(engine.HostTensor.from_dlpack(p).to_hbm(device), len(p), alloc.take(6))
            for p in prompts]
    steps = 16
    out = serving.prefill(model, cache, seqs, list(range(len(seqs))))
    tokens = [[t] for t in out.to_host().numpy().tolist()]
    for _ in range(steps):
        out = serving.decode(model, cache, seqs)
        for i, t in enumerate(out.to_host().numpy().tolist()):
            tokens[i].append(t)
    device.synchronize()
    # Greedy continuation of the dense forward, token by token.
    for i, p in enumerate(prompts):
        seq = p.clone()
        for step in range(steps + 1):
            logits = dense.forward(w, cfg, seq)[-1]
            top = torch.topk(logits, 2).values
            pick = tokens[i][step]
            # The engine's token must be the dense argmax, or within 1e-2 of it (BF16 rounding
            # differences can swap near-ties).
            assert logits[pick] >= top[0] - 1e-2 * max(1.0, abs(top[0].item())), (i, step)
            seq = torch.cat([seq, torch.tensor([pick], dtype=torch.int32)])


def test_refusals_match_reference_messages():
    engine, cfg, device, model = _build()
    from furiosa_opt_engine import decoder as dec

    cache = dec.Cache(model.cache, 8)
    ids = engine.HostTensor([1, 2, 3]).to_hbm(device)
    cases = [
        ([], "call has no requests"),
        ([dec.Request([[0]], 14, ids)], "request has fewer blocks than its positions need"),
        ([dec.Request([[9]], 0, ids)], "block ID is outside the cache"),
        ([dec.Request([[0]], 0, ids, range(2, 5))], "kept rows lie outside the appended rows"),
        ([dec.Request([[0]], 0, ids), dec.Request([[0]], 0, ids)], "two appended positions share a cache slot"),
    ]
    for reqs, msg in cases:
        with pytest.raises(ValueError, match=msg):
            model.forward(reqs, cache)
    with pytest.raises(NotImplementedError, match="explicit positions are not served"):
        model.forward([dec.Request([[0]], 0, ids, positions=ids)], cache)


@pytest.mark.parametrize("name", ["tiny-qwen3", "tiny-qwen3-moe"])
def test_load_checkpoint_strictly_and_decode(tmp_path, name):
    """A synthetic HF checkpoint through Checkpoint -> LoadOptions.load: the loaded decoder's
    greedy continuation agrees with the dense forward of the checkpoint's own weights."""
    import furiosa_opt_engine as engine
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get(name)
    hf = synthetic.write(str(tmp_path / "m"), cfg, seed=5, std=0.05, shards=2)
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    ck = engine.Checkpoint(str(tmp_path / "m"))
    device = engine.Device(engine.Placement([0], range(8)))
    model = engine.LoadOptions().load(ck, device)
    assert type(model).__name__ == "ForCausalLM" and model.size == "custom"
    assert model.cache.pools[0].block == 16
    cache = dec.Cache(model.cache, 32)
    alloc = serving.BlockAllocator(32)
    gen = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg["vocab"], (21,), generator=gen, dtype=torch.int32)
    seqs = [serving.Sequence(engine.HostTensor.from_dlpack(prompt).to_hbm(device), 21, alloc.take(4))]
    toks = [serving.prefill(model, cache, seqs, [0]).to_host().numpy()[0]]
    for _ in range(8):
        toks.append(serving.decode(model, cache, seqs).to_host().numpy()[0])
    seq = prompt.clone()
    for t in toks:
        logits = dense.forward(w, cfg, seq)[-1]
        tol = 5e-2 if cfg.get("experts") else 1e-2
        assert logits[int(t)] >= logits.max() - tol * max(1.0, abs(logits.max().item()))
        seq = torch.cat([seq, torch.tensor([int(t)], dtype=torch.int32)])


def test_load_refuses_a_missing_tensor(tmp_path):
    import os

    import furiosa_opt_engine as engine
    from safetensors.torch import load_file, save_file
    from furiosa_opt_models_b200.models import synthetic

    synthetic.write(str(tmp_path / "m"), "tiny-qwen3")
    path = str(tmp_path / "m" / "model.safetensors")
    w = load_file(path)
    del w["model.layers.1.mlp.down_proj.weight"]
    w["model.extra.weight"] = torch.zeros(4, dtype=torch.bfloat16)
    save_file(w, path)
    device = engine.Device(engine.Placement([0], range(8)))
    with pytest.raises(ValueError, match="missing tensors: model.layers.1.mlp.down_proj.weight"):
        engine.LoadOptions().load(engine.Checkpoint(str(tmp_path / "m")), device)


@pytest.mark.parametrize("fmt", ["fp8_block", "nvfp4_a4", "nvfp4"])
def test_quantized_decoder_matches_dense_contract(fmt):
    """Quantized projections (W8A8, W4A4, W4A16) through the engine against the dense forward
    that applies the same contracts (input quantization included) in FP32."""
    engine, cfg, device, model = _build(weight_format=fmt)
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import dense

    w = _weights(model)
    assert not isinstance(w["layers.0.qkv"], torch.Tensor)
    lengths = [5, 19, 40]
    gen = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen, dtype=torch.int32) for n in lengths]
    cache = dec.Cache(model.cache, 32)
    alloc = serving.BlockAllocator(32)
    seqs = [serving.Sequence(engine.HostTensor.from_dlpack(p).to_hbm(device), len(p), alloc.take(4))
            for p in prompts]
    steps = 4
    out = serving.prefill(model, cache, seqs, list(range(len(seqs))))
    tokens = [[t] for t in out.to_host().numpy().tolist()]
    for _ in range(steps):
        out = serving.decode(model, cache, seqs)
        for i, t in enumerate(out.to_host().numpy().tolist()):
            tokens[i].append(t)
    device.synchronize()
    for i, p in enumerate(prompts):
        seq = p.clone()
        for step in range(steps + 1):
            logits = dense.forward(w, cfg, seq)[-1]
            top = torch.topk(logits, 2).values
            pick = tokens[i][step]
            # Input quantization turns a rounding difference upstream into a whole code step (a
            # third of a value for E2M1), so the engine's token may trail the dense maximum.
            tol = 0.15 if fmt == "nvfp4_a4" else 5e-2
            assert logits[pick] >= top[0] - tol * max(1.0, abs(top[0].item())), (fmt, i, step)
            seq = torch.cat([seq, torch.tensor([pick], dtype=torch.int32)])


@pytest.mark.parametrize("graphs", [True, False])
def test_moe_decoder_matches_dense(graphs):
    """A tiny Qwen3-MoE decoder (16 experts, top-4) through the engine's routing, grouped expert
    GEMMs and choice-order combine against the dense forward of the same weights."""
    engine, cfg, device, model = _build("tiny-qwen3-moe")
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import dense

    model.set_graphs(graphs)
    w = _weights(model)
    lengths = [9, 30, 64]
    gen = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen, dtype=torch.int32) for n in lengths]
    cache = dec.Cache(model.cache, 32)
    alloc = serving.BlockAllocator(32)
    seqs = [serving.Sequence(engine.HostTensor.from_dlpack(p).to_hbm(device), len(p), alloc.take(6))
            for p in prompts]
    steps = 6
    out = serving.prefill(model, cache, seqs, list(range(len(seqs))))
    tokens = [[t] for t in out.to_host().numpy().tolist()]
    for _ in range(steps):
        out = serving.decode(model, cache, seqs)
        for i, t in enumerate(out.to_host().numpy().tolist()):
            tokens[i].append(t)
    device.synchronize()
    for i, p in enumerate(prompts):
        seq = p.clone()
        for step in range(steps + 1):
            logits = dense.forward(w, cfg, seq)[-1]
            top = torch.topk(logits, 2).values
            pick = tokens[i][step]
            # A router logit one BF16 step apart can reorder or swap a selected expert.
            assert logits[pick] >= top[0] - 5e-2 * max(1.0, abs(top[0].item())), (i, step)
            seq = torch.cat([seq, torch.tensor([pick], dtype=torch.int32)])


@pytest.mark.parametrize("granularity", ["fp8_per_channel", "fp8_per_tensor"])
def test_load_time_fp8_quantization(tmp_path, granularity):
    """A BF16 checkpoint quantized to FP8 at load (LoadOptions.quantization): greedy decoding
    agrees with the dense forward of the loaded codes and scales (restored to BF16, W8A16)."""
    import furiosa_opt_engine as engine
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-qwen3")
    synthetic.write(str(tmp_path / "m"), cfg, seed=8, std=0.05)
    ck = engine.Checkpoint(str(tmp_path / "m"))
    device = engine.Device(engine.Placement([0], range(8)))
    model = engine.LoadOptions().quantization(granularity).load(ck, device)
    w = _weights(model)
    assert w["layers.0.qkv"].format == "fp8_rows"
    if granularity == "fp8_per_tensor":
        assert w["layers.0.qkv"].scales.unique().numel() == 1
    cache = dec.Cache(model.cache, 32)
    alloc = serving.BlockAllocator(32)
    gen = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, cfg["vocab"], (19,), generator=gen, dtype=torch.int32)
    seqs = [serving.Sequence(engine.HostTensor.from_dlpack(prompt).to_hbm(device), 19, alloc.take(4))]
    toks = [serving.prefill(model, cache, seqs, [0]).to_host().numpy()[0]]
    for _ in range(6):
        toks.append(serving.decode(model, cache, seqs).to_host().numpy()[0])
    seq = prompt.clone()
    for t in toks:
        logits = dense.forward(w, cfg, seq)[-1]
        assert logits[int(t)] >= logits.max() - 1e-2 * max(1.0, abs(logits.max().item()))
        seq = torch.cat([seq, torch.tensor([int(t)], dtype=torch.int32)])


def test_lora_adapters_in_two_slots(tmp_path):
    """Two PEFT LoRA adapters in the two slots of one call, and a request with none: each
    request's greedy tokens agree with the dense forward of its merged weights."""
    import json as _json

    import furiosa_opt_engine as engine
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-qwen3")
    device = engine.Device(engine.Placement([0], range(8)))
    model = engine._native._synthetic_decoder(device, cfg, seed=7, std=0.05, adapters=2)
    spec = model.adapters
    assert spec is not None and spec.RANK == 32 and spec.SLOTS == 2
    base = _weights(model)
    adapters, merged = [], []
    for i, (r, alpha) in enumerate([(8, 16.0), (16, 8.0)]):
        d = tmp_path / f"lora{i}"
        lora = synthetic.write_lora(str(d), cfg, r=r, alpha=alpha, seed=i + 1)
        with open(d / "adapter_config.json") as f:
            ck = engine.Checkpoint(str(d), config=_json.load(f))
        adapters.append(dec.Adapter(spec, ck))
        merged.append(synthetic.merge_lora(base, cfg, lora, r, alpha))
    gen = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen, dtype=torch.int32) for n in (9, 21, 14)]
    slots = [0, 1, None]
    cache = dec.Cache(model.cache, 32)
    alloc = serving.BlockAllocator(32)
    seqs = [serving.Sequence(engine.HostTensor.from_dlpack(p).to_hbm(device), len(p), alloc.take(4)) for p in prompts]
    reqs = [dec.Request([s.blocks], 0, s.prompt, dec.Keep.LAST, adapter=slot) for s, slot in zip(seqs, slots)]
    out = model.forward(reqs, cache, adapters).to_host().numpy().tolist()
    device.synchronize()
    for p, t, slot in zip(prompts, out, slots):
        w = base if slot is None else merged[slot]
        logits = dense.forward(w, cfg, p)[-1]
        assert logits[t] >= logits.max() - 1e-2 * max(1.0, abs(logits.max().item())), slot
    # A request naming an empty slot is refused.
    with pytest.raises(ValueError):
        model.forward([dec.Request([seqs[0].blocks], 0, seqs[0].prompt, dec.Keep.LAST, adapter=1)], cache,
                      [adapters[0], None])


def test_mixtral_checkpoint_loads_strictly_and_matches_dense(tmp_path):
    """A tiny Mixtral checkpoint (block_sparse_moe names, 8 experts, top-2 renormalised) loads
    through LoadOptions as mixtral.ForCausalLM and decodes the dense forward's greedy tokens."""
    import furiosa_opt_engine as engine
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-mixtral")
    hf = synthetic.write(str(tmp_path / "m"), cfg, seed=5, std=0.05)
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    device = engine.Device(engine.Placement([0], range(8)))
    model = engine.LoadOptions().load(engine.Checkpoint(str(tmp_path / "m")), device)
    assert isinstance(model, engine.mixtral.ForCausalLM)
    gen = torch.Generator().manual_seed(8)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen, dtype=torch.int32) for n in (6, 25, 48)]
    cache = dec.Cache(model.cache, 32)
    alloc = serving.BlockAllocator(32)
    seqs = [serving.Sequence(engine.HostTensor.from_dlpack(p).to_hbm(device), len(p), alloc.take(6))
            for p in prompts]
    steps = 5
    out = serving.prefill(model, cache, seqs, list(range(len(seqs))))
    tokens = [[t] for t in out.to_host().numpy().tolist()]
    for _ in range(steps):
        out = serving.decode(model, cache, seqs)
        for i, t in enumerate(out.to_host().numpy().tolist()):
            tokens[i].append(t)
    device.synchronize()
    for i, p in enumerate(prompts):
        seq = p.clone()
        for step in range(steps + 1):
            logits = dense.forward(w, cfg, seq)[-1]
            top = torch.topk(logits, 2).values
            pick = tokens[i][step]
            assert logits[pick] >= top[0] - 5e-2 * max(1.0, abs(top[0].item())), (i, step)
            seq = torch.cat([seq, torch.tensor([pick], dtype=torch.int32)])


def test_launch_program_is_a_module_tree():
    """The decoder's launch program is composed of modules: per-layer attention and feed-forward
    blocks under a Layers combinator, the experts block in place of the MLP for a MoE family."""
    _, _, _, dense_model = _build()
    tree = dense_model.program
    assert tree.splitlines()[0] == "qwen3 decoder"
    assert "Layers x2" in tree and "GateUp" in tree and "Choice decode rows" in tree and "Experts" not in tree
    _, _, _, moe = _build("tiny-qwen3-moe")
    assert "Experts" in moe.program and "GateUp" not in moe.program


def test_static_fp8_checkpoint_matches_its_restored_weights(tmp_path):
    """A static per-tensor FP8 checkpoint (Mistral NeMo FP8 style: E4M3 codes, one weight_scale
    and one input_scale a projection) loads as mistral.ForCausalLM with FP8 precision and decodes
    the dense forward's greedy tokens of the restored weights bf16(code * weight_scale)."""
    import json
    import os

    from safetensors.torch import save_file

    import furiosa_opt_engine as engine
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-mistral")
    hf = synthetic.hf_weights(cfg, seed=9, std=0.05)
    q = synthetic.quantize_static_fp8(hf)
    d = str(tmp_path / "m")
    os.makedirs(d)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(dict(synthetic.hf_config(cfg), quantization_config=synthetic.STATIC_FP8), f)
    save_file(q, os.path.join(d, "model.safetensors"))
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, synthetic.dequantize_static_fp8(q)).items()}
    device = engine.Device(engine.Placement([0], range(8)))
    model = engine.LoadOptions().load(engine.Checkpoint(d), device)
    assert isinstance(model, engine.mistral.ForCausalLM) and model.precision == "float8_e4m3fn"
    gen = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen, dtype=torch.int32) for n in (9, 40)]
    cache = dec.Cache(model.cache, 16)
    alloc = serving.BlockAllocator(16)
    seqs = [serving.Sequence(engine.HostTensor.from_dlpack(p).to_hbm(device), len(p), alloc.take(5)) for p in prompts]
    out = serving.prefill(model, cache, seqs, [0, 1])
    tokens = [[t] for t in out.to_host().numpy().tolist()]
    for _ in range(4):
        out = serving.decode(model, cache, seqs)
        for i, t in enumerate(out.to_host().numpy().tolist()):
            tokens[i].append(t)
    for i, p in enumerate(prompts):
        seq = p.clone()
        for step in range(5):
            logits = dense.forward(w, cfg, seq)[-1]
            top = torch.topk(logits, 2).values
            pick = tokens[i][step]
            assert logits[pick] >= top[0] - 1e-2 * max(1.0, abs(top[0].item())), (i, step)
            seq = torch.cat([seq, torch.tensor([pick], dtype=torch.int32)])
