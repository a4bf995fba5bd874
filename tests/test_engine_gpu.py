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
    from furiosa_opt_models_b200.utils import devmem

    return {k: v.float().cpu() for k, v in devmem.weights(model).items()}


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
