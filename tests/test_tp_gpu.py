"""Tensor parallelism on 2+ GPUs. Numerics: a base-model checkpoint loaded at TP=N through the public
API gives final hidden rows that match TP=1 and the dense FP32 forward of the same weights within a
BF16 bound, and the same bits on a second run. Tokens: the same synthetic decoder (identical
logical weights at every split) decodes the same greedy tokens at TP=1 and TP=N. Each rank is a
process of its own GPU; the fused collectives spin only on peers of other GPUs."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, "tests", "workers", "tp_parity.py")


def _torchrun(world: int, worker: str, args: list, **extra_env) -> None:
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1", **extra_env)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", "--master-port=29533", worker, *args]
    subprocess.run(cmd, check=True, env=env, cwd=ROOT)


def _run(world: int, out: str, model: str, steps: int, **extra_env) -> list:
    _torchrun(world, WORKER, [out, model, str(steps)], **extra_env)
    with open(out) as f:
        return json.load(f)


def _base_model(directory: str, steps: int):
    """A Qwen3Model checkpoint (hidden rows out) of a geometry that splits over 2-8 chips, its
    workload, and the dense FP32 forward's final-normed rows of every fed token."""
    from safetensors.torch import save_file

    from furiosa_opt_models_b200.models import configs, dense, synthetic

    cfg = configs.get("tiny-qwen3-tp", tied=False)
    hf = synthetic.hf_weights(cfg, seed=11, std=0.05)
    w = {k: v.float() for k, v in synthetic.engine_weights(cfg, hf).items()}
    os.makedirs(directory, exist_ok=True)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(dict(synthetic.hf_config(cfg), architectures=["Qwen3Model"]), f)
    save_file({k: v for k, v in hf.items() if k != "lm_head.weight"}, os.path.join(directory, "model.safetensors"))
    gen = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen, dtype=torch.int32) for n in (5, 16, 37, 200)]
    fed = [torch.randint(0, cfg["vocab"], (steps,), generator=gen, dtype=torch.int32).tolist() for _ in prompts]
    torch.save({"prompts": prompts, "fed": fed}, os.path.join(directory, "workload.pt"))
    want = [dense.forward(w, cfg, torch.cat([p, torch.tensor(f, dtype=torch.int32)]), head=False)
            for p, f in zip(prompts, fed)]
    return prompts, want


def _close(got: torch.Tensor, want: torch.Tensor, rel: float) -> None:
    err = (got - want).abs().max().item()
    assert err <= rel * max(1.0, want.abs().max().item()), err
    assert torch.nn.functional.cosine_similarity(got, want, dim=-1).min().item() > 0.999


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["one-shot", "two-shot"])
def test_tp_hidden_rows_match_one_gpu_and_dense(world, mode, tmp_path):
    """Final hidden rows of a prompt call (every row kept) and 6 decode calls at TP=N against TP=1
    and the dense FP32 forward; a second TP=N run gives the same bits (rank-ordered FP32 sums)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    steps = 6
    ckpt = str(tmp_path / "ckpt")
    prompts, want = _base_model(ckpt, steps)
    worker = os.path.join(ROOT, "tests", "workers", "tp_hidden.py")
    env = {"FOA_TP_ONESHOT_BYTES": "0"} if mode == "two-shot" else {"FOA_TP_ONESHOT_BYTES": str(1 << 30)}
    _torchrun(1, worker, [str(tmp_path / "one.pt"), ckpt, str(steps)])
    _torchrun(world, worker, [str(tmp_path / "many.pt"), ckpt, str(steps)], **env)
    _torchrun(world, worker, [str(tmp_path / "again.pt"), ckpt, str(steps)], **env)
    one, many, again = (torch.load(str(tmp_path / f"{n}.pt")) for n in ("one", "many", "again"))
    assert all(torch.equal(a, b) for a, b in zip(many, again)), "TP=N is not deterministic run to run"
    # Prompt rows, then one row a sequence a decode step, against the dense rows of the same positions.
    offsets = [0]
    for p in prompts:
        offsets.append(offsets[-1] + len(p))
    for i, p in enumerate(prompts):
        rows = [many[0][offsets[i] : offsets[i + 1]]] + [many[1 + s][i : i + 1] for s in range(steps)]
        got = torch.cat(rows)
        _close(got, want[i], 0.03)
        ref = torch.cat([one[0][offsets[i] : offsets[i + 1]]] + [one[1 + s][i : i + 1] for s in range(steps)])
        _close(got, ref, 0.03)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_batch_invariant_tp_is_bitwise_repeatable(tmp_path):
    """A batch-invariant load at TP=2 gives bitwise the same hidden rows on two runs."""
    steps = 4
    ckpt = str(tmp_path / "ckpt")
    _base_model(ckpt, steps)
    worker = os.path.join(ROOT, "tests", "workers", "tp_hidden.py")
    for name in ("a", "b"):
        _torchrun(2, worker, [str(tmp_path / f"{name}.pt"), ckpt, str(steps), "invariant"])
    a, b = torch.load(str(tmp_path / "a.pt")), torch.load(str(tmp_path / "b.pt"))
    assert all(torch.equal(x, y) for x, y in zip(a, b))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["one-shot", "two-shot"])
def test_tp_matches_single_gpu(world, mode, tmp_path):
    """`two-shot` forces every all-reduce through the reduce-scatter path (each rank reduces the
    rows of its slice from every rank's partial; owners store the normed rows into every rank)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    one = _run(1, str(tmp_path / "tp1.json"), "tiny-qwen3-tp", 12)
    env = {"FOA_TP_ONESHOT_BYTES": "0"} if mode == "two-shot" else {"FOA_TP_ONESHOT_BYTES": str(1 << 30)}
    many = _run(world, str(tmp_path / f"tp{world}.json"), "tiny-qwen3-tp", 12, **env)
    # Greedy tokens agree (the FP32 partial sums are added in another grouping, so a near-tie may
    # flip a token late in a sequence; the first tokens must match exactly).
    assert [t[:4] for t in one] == [t[:4] for t in many]
    agree = sum(a == b for s1, s2 in zip(one, many) for a, b in zip(s1, s2))
    total = sum(len(s) for s in one)
    assert agree >= 0.9 * total, (agree, total)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", [2, 4, 8])
def test_expert_parallel_matches_single_gpu(world, tmp_path):
    """Qwen3-MoE with experts sharded over `world` ranks (the combine reads peers' expert rows over
    NVLink) against one GPU holding every expert."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    one = _run(1, str(tmp_path / "ep1.json"), "tiny-qwen3-moe", 12)
    many = _run(world, str(tmp_path / f"ep{world}.json"), "tiny-qwen3-moe", 12)
    # Top-k routing turns the different FP32 grouping of the attention projection's cross-rank sum
    # into a different expert choice at a near-tie, after which a sequence follows another greedy
    # path; the first two tokens of every sequence must match and most sequences must match whole.
    assert [t[:2] for t in one] == [t[:2] for t in many]
    whole = sum(s1 == s2 for s1, s2 in zip(one, many))
    assert whole >= len(one) - 1, (one, many)
    # The expert-parallel path is deterministic: a second run gives the same tokens.
    again = _run(world, str(tmp_path / f"ep{world}b.json"), "tiny-qwen3-moe", 12)
    assert again == many


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_all_gather_and_exchange(world, tmp_path):
    """The reference's AllGather (parts in rank order) and Exchange (rank t takes rows t*S.. of
    every rank's columns) of BF16 rows over the peer heap, between decoder calls, on every rank."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = str(tmp_path / "rows")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1")
    subprocess.run(["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                    f"--nproc-per-node={world}", "--master-addr=127.0.0.1", "--master-port=29534",
                    os.path.join(ROOT, "tests", "workers", "tp_rows.py"), out], check=True, env=env, cwd=ROOT)
    for r in range(world):
        with open(f"{out}.{r}") as f:
            results = json.load(f)
        assert results and all(results.values()), (r, results)
