"""The SGLang plugin's runner on SGLang-shaped batches (a req_to_token slot table with 16-token
pages, extend then decode batches) through the engine, against the dense forward."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_extend_and_decode_batches_match_dense():
    import furiosa_opt_engine as engine
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200.models import configs, dense
    from furiosa_opt_sglang.runner import Runner

    from test_engine_gpu import _weights

    cfg = configs.get("tiny-qwen3")
    device = engine.Device(engine.Placement([0], range(8)))
    model = engine._native._synthetic_decoder(device, cfg, seed=9, std=0.05)
    cache = dec.Cache(model.cache, 64)
    runner = Runner(model, device, cache)
    w = _weights(model)
    gen = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen).tolist() for n in (12, 35)]
    # Pool rows 0 and 1; their slots fill pages 5.. and 20.. (page = slot // 16).
    req_to_token = torch.zeros(2, 256, dtype=torch.int64)
    req_to_token[0] = torch.arange(5 * 16, 5 * 16 + 256)
    req_to_token[1] = torch.arange(20 * 16, 20 * 16 + 256)
    table = req_to_token.tolist()
    flat = prompts[0] + prompts[1]
    first = runner.extend([0, 1], [12, 35], [0, 0], [12, 35], flat, table)
    seqs = [p + [t] for p, t in zip(prompts, first)]
    for _ in range(5):
        nxt = runner.decode([0, 1], [len(s) for s in seqs], [s[-1] for s in seqs], table)
        seqs = [s + [t] for s, t in zip(seqs, nxt)]
    device.synchronize()
    for p, s in zip(prompts, seqs):
        for i in range(len(p), len(s)):
            logits = dense.forward(w, cfg, torch.tensor(s[:i], dtype=torch.int32))[-1]
            assert logits[s[i]] >= logits.max() - 1e-2 * max(1.0, abs(logits.max().item()))
