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


def _batch(slots, seq_lens, ids, extend_lens=None):
    from types import SimpleNamespace

    class Mode:
        def is_extend(self):
            return extend_lens is not None

        def is_decode(self):
            return extend_lens is None

    info = SimpleNamespace(is_all_greedy=True, grammars=None, logit_bias=None, acc_additive_penalties=None,
                           acc_scaling_penalties=None, has_custom_logit_processor=False)
    return SimpleNamespace(forward_mode=Mode(), reqs=[object() for _ in slots], req_pool_indices=torch.tensor(slots),
                           seq_lens=torch.tensor(seq_lens), extend_lens=extend_lens, input_ids=torch.tensor(ids),
                           decoding_reqs=None, sampling_info=info, return_logprob=False)


def test_overlap_steps_match_synchronous_steps():
    """Scheduled steps with SGLang's overlap schedule (decode rows read the previous step's tokens
    on the device; the batch IDs are placeholders) give the tokens of the synchronous runner."""
    import furiosa_opt_engine as engine
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200.models import configs
    from furiosa_opt_sglang.runner import Runner

    cfg = configs.get("tiny-qwen3")
    device = engine.Device(engine.Placement([0], range(8)))
    model = engine._native._synthetic_decoder(device, cfg, seed=9, std=0.05)
    gen = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen).tolist() for n in (12, 35)]
    req_to_token = torch.zeros(2, 256, dtype=torch.int64)
    req_to_token[0] = torch.arange(5 * 16, 5 * 16 + 256)
    req_to_token[1] = torch.arange(20 * 16, 20 * 16 + 256)
    table = req_to_token.tolist()

    sync = Runner(model, device, dec.Cache(model.cache, 64))
    first = sync.extend([0, 1], [12, 35], [0, 0], [12, 35], prompts[0] + prompts[1], table)
    want = [[t] for t in first]
    for _ in range(5):
        nxt = sync.decode([0, 1], [len(p) + len(w) for p, w in zip(prompts, want)], [w[-1] for w in want], table)
        want = [w + [t] for w, t in zip(want, nxt)]

    runner = Runner(model, device, dec.Cache(model.cache, 64))
    pending = runner.issue(_batch([0, 1], [12, 35], prompts[0] + prompts[1], extend_lens=[12, 35]), req_to_token)
    got = [[], []]
    for i in range(5):
        lens = [12 + i + 1, 35 + i + 1]
        result = runner.issue(_batch([0, 1], lens, [0, 0]), req_to_token)
        pending.collect()
        got = [g + [int(t)] for g, t in zip(got, pending.next_token_ids.tolist())]
        pending = result
    pending.collect()
    got = [g + [int(t)] for g, t in zip(got, pending.next_token_ids.tolist())]
    assert got == want


def test_host_tier_round_trip_through_the_engine_cache():
    """Pages backed up to the host tier, overwritten on the device, and loaded back layer by layer
    come back bit for bit."""
    import numpy as np

    import furiosa_opt_engine as engine
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200.models import configs
    from furiosa_opt_sglang import hicache

    cfg = configs.get("tiny-qwen3")
    device = engine.Device(engine.Placement([0], range(8)))
    model = engine._native._synthetic_decoder(device, cfg, seed=9, std=0.05)
    cache = dec.Cache(model.cache, 32)
    page = int(cache.spec.pools[0].bytes)
    rng = np.random.default_rng(3)
    before = []
    for layer in cache.layers:
        data = rng.integers(0, 255, size=len(layer), dtype=np.uint8)
        engine.HostBuffer(data).to_hbm(layer).wait()
        before.append(data)
    tier = hicache.HostTier(engine, cache, pages=8)
    tier.backup(torch.arange(16 * 4, 16 * 7), torch.arange(16 * 1, 16 * 4))  # blocks 4..6 -> pages 1..3
    tier.wait()
    for layer in cache.layers:
        engine.HostBuffer(np.zeros(3 * page, dtype=np.uint8)).to_hbm(layer.slice(4 * page, 3 * page)).wait()
    for i in range(len(cache.layers)):
        tier.load(torch.arange(16 * 1, 16 * 4), torch.arange(16 * 10, 16 * 13), i)  # pages 1..3 -> blocks 10..12
    for i in range(len(cache.layers)):
        tier.load(torch.arange(16 * 1, 16 * 4), torch.arange(16 * 4, 16 * 7), i)  # and back to 4..6
    tier.wait()
    for layer, data in zip(cache.layers, before):
        host = engine.HostBuffer(len(layer))
        layer.to_host(host).wait()
        got = np.frombuffer(memoryview(host), dtype=np.uint8)
        assert np.array_equal(got[4 * page : 7 * page], data[4 * page : 7 * page])
        assert np.array_equal(got[10 * page : 13 * page], data[4 * page : 7 * page])
        assert np.array_equal(got[: 4 * page], data[: 4 * page])


@pytest.mark.parametrize("proposer", ["ngram", "draft_same", "draft_other"])
def test_speculative_steps_commit_greedy_tokens(proposer):
    """SGLang's speculative schedule through the engine: n-gram drafts, a draft model equal to the
    target (every draft accepted) and an unrelated one (most rejected); every committed token is the
    dense forward's greedy token."""
    from types import SimpleNamespace

    import furiosa_opt_engine as engine
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200.models import configs, dense
    from furiosa_opt_sglang import speculative
    from furiosa_opt_sglang.runner import Runner

    from test_engine_gpu import _weights

    cfg = configs.get("tiny-qwen3")
    device = engine.Device(engine.Placement([0], range(8)))
    model = engine._native._synthetic_decoder(device, cfg, seed=9, std=0.05)
    runner = Runner(model, device, dec.Cache(model.cache, 64))
    if proposer == "ngram":
        propose = speculative.Ngram(k=3)
    else:
        draft = engine._native._synthetic_decoder(device, cfg, seed=9 if proposer == "draft_same" else 4, std=0.05)
        propose = speculative.DraftModel(draft, dec.Cache(draft.cache, 64), k=3)
    spec = speculative.Speculation(propose, width=4)
    gen = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen).tolist() for n in (12, 35)]
    prompts[0] = (prompts[0][:6] * 2)  # a repeat for the n-gram drafts to find
    req_to_token = torch.zeros(2, 256, dtype=torch.int64)
    req_to_token[0] = torch.arange(5 * 16, 5 * 16 + 256)
    req_to_token[1] = torch.arange(20 * 16, 20 * 16 + 256)
    table = req_to_token.tolist()
    reqs = [SimpleNamespace(rid=str(i), origin_input_ids=p, output_ids=[]) for i, p in enumerate(prompts)]
    extend = _batch([0, 1], [12, 35], prompts[0] + prompts[1], extend_lens=[12, 35])
    extend.reqs = reqs
    first = speculative.forward(runner, spec, extend, table, context=256)
    for r, t in zip(reqs, first.next_token_ids.view(2, 4)[:, 0].tolist()):
        r.output_ids.append(int(t))
    accepted = 0
    while min(len(r.output_ids) for r in reqs) < 10:
        b = _batch([0, 1], [len(r.origin_input_ids) + len(r.output_ids) - 1 for r in reqs], [0, 0])
        b.reqs = reqs
        result = speculative.forward(runner, spec, b, table, context=256)
        packed = result.next_token_ids.view(2, 4)
        for i, r in enumerate(reqs):
            n = int(result.accept_lens[i])
            accepted += n - 1
            r.output_ids += packed[i, :n].tolist()
    device.synchronize()
    w = _weights(model)
    for r in reqs:
        s = r.origin_input_ids + r.output_ids
        for i in range(len(r.origin_input_ids), len(s)):
            logits = dense.forward(w, cfg, torch.tensor(s[:i], dtype=torch.int32))[-1]
            assert logits[s[i]] >= logits.max() - 1e-2 * max(1.0, abs(logits.max().item()))
    if proposer == "draft_same":
        assert accepted > 0
