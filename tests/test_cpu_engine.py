"""The tiny Qwen3 CPU configuration: the paged FP32 engine path against the dense FP32 PyTorch
forward: one prefill call of prompts 7/16/33/64, then 16 greedy decode calls, logits compared."""

import torch

from furiosa_opt_models_b200.models import configs, cpu_engine, dense, synthetic


def test_tiny_qwen3_paged_matches_dense():
    cfg = configs.get("tiny-qwen3")
    hf = synthetic.hf_weights(cfg, seed=0, std=0.02)
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    model = cpu_engine.CpuDecoder(cfg, w, blocks=64)
    gen = torch.Generator().manual_seed(0)
    lengths = [7, 16, 33, 64]
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen, dtype=torch.int32) for n in lengths]
    free = list(range(64))
    blocks = [[free.pop(0) for _ in range(6)] for _ in lengths]
    seqs = [p.clone() for p in prompts]
    logits = model.forward([cpu_engine.Request(b, 0, p) for b, p in zip(blocks, prompts)])
    for step in range(17):
        for i, seq in enumerate(seqs):
            ref = dense.forward(w, cfg, seq, round_bf16=False)[-1]
            assert torch.allclose(logits[i], ref, atol=1e-4, rtol=1e-4), (step, i)
        nxt = logits.argmax(-1).to(torch.int32)
        if step == 16:
            break
        reqs = [cpu_engine.Request(b, len(s), nxt[i : i + 1]) for i, (b, s) in enumerate(zip(blocks, seqs))]
        seqs = [torch.cat([s, nxt[i : i + 1]]) for i, s in enumerate(seqs)]
        logits = model.forward(reqs)
