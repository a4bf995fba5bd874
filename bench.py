"""Serving benchmark: output tokens/s at fixed concurrency, with p50 TTFT and TPOT.

One "step" is one wave of the BASELINE workload: `concurrency` synthetic requests of `input_len`
uniform-random prompt tokens each, prefilled in calls of at most `rows` rows, then greedily decoded
to `output_len` output tokens (the prefill yields the first). The model is the named architecture
with random-init N(0, 0.02) BF16 weights. On N GPUs the wave runs tensor-parallel over N ranks
(one process per GPU, launched by torch.distributed.run).

Timing: W untimed warm-up waves, then K timed waves between a barrier and a device sync on both
sides, measured with CUDA events on the engine's stream; the reported time is the max over ranks.
The e2e arm runs the same waves through the public API with every step's inputs copied from pinned
host memory and every step's output tokens read back to the host.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference|baseline|vllm]

`--impl baseline` runs the waves on eager PyTorch (cuBLAS, SDPA, NCCL); `--impl vllm` on stock
vLLM, the library serving stack of this image.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "output tok/s at fixed concurrency, p50 TTFT/TPOT, TP=1/2/4/8, device-timed max/rank"


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference", "baseline", "vllm"])
    p.add_argument("--model", default="qwen3-1.7b")
    p.add_argument("--concurrency", type=int, default=64)
    p.add_argument("--input-len", type=int, default=1024)
    p.add_argument("--output-len", type=int, default=128)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-graphs", action="store_true")
    return p.parse_args()


def reference_arm(args) -> None:
    reason = (
        "the reference (furiosa-ai/furiosa-opt-models) does not install here: its root is a uv "
        "workspace with no build backend and its engine wheel needs maturin, nightly Rust and "
        "cargo-furiosa-opt to build Rust/VISA kernels for FuriosaAI RNGD NPUs; it has no CUDA path"
    )
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        self.file.flush()
        rows = []
        try:
            with open(self.file.name) as f:
                for line in f:
                    parts = [x.strip() for x in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
        finally:
            os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
            "reasons": reasons,
            "samples": len(rows),
        }


def baseline_arm(args, torch, dist, world, rank, local) -> None:
    """The same waves on stock PyTorch (cuBLAS matmuls, fused SDPA attention over a contiguous KV
    cache, NCCL all-reduce), eager: the library baseline the engine is compared with."""
    from furiosa_opt_models_b200.models import configs
    from furiosa_opt_models_b200.models.baseline import Baseline

    cfg = configs.get(args.model)
    if cfg.get("experts") or cfg.get("weight_format", "bf16") != "bf16":
        if rank == 0:
            print(json.dumps({"impl": "baseline", "unavailable": "the PyTorch baseline covers dense BF16 decoders"}))
        return
    model = Baseline(cfg, tp=world, rank=rank)
    B, L = args.concurrency, args.input_len + args.output_len
    model.allocate(B, L)
    gen = torch.Generator().manual_seed(1234)
    prompts = torch.randint(0, cfg["vocab"], (B, args.input_len), generator=gen, dtype=torch.int64).cuda()
    chunk = max(1, 8192 // args.input_len)

    def wave():
        toks = []
        for b0 in range(0, B, chunk):  # prefill in chunks of about 8192 rows, as the engine's calls
            toks.append(model.forward(prompts[b0:b0 + chunk], 0, b0))
        last = torch.cat(toks)[:, None]
        for step in range(args.output_len - 1):
            last = model.forward(last, args.input_len + step)[:, None]

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        wave()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    with sampler:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            wave()
        t1.record()
        torch.cuda.synchronize()
    barrier()
    ms = torch.tensor([t0.elapsed_time(t1) / args.steps], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = ms.item()
    if rank == 0:
        print(json.dumps({
            "impl": "baseline", "metric": METRIC,
            "value": round(B * args.output_len / (ms / 1e3), 1), "unit": "output tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
            "data": "synthetic: uniform-random prompt token IDs; random-init N(0,0.02) weights",
            "config": {"model": f"{args.model} (shape of the named checkpoint)", "global_batch": B,
                       "seq_len": L, "parallelism": f"tp{world}",
                       "stack": "PyTorch eager: cuBLAS matmul, fused SDPA over a contiguous KV cache, NCCL all-reduce"},
            "clocks": sampler.summary(),
        }), flush=True)


def vllm_arm(args, world: int, rank: int, local: int) -> None:
    """The same waves through stock vLLM (its own B200 kernels, CUDA graphs, NCCL and custom
    all-reduce), none of this repository's kernels or engine on the path: the library serving
    stack the engine is compared with. Weights are vLLM's dummy initialisation of the named
    geometry (no checkpoint); at N > 1 every torchrun rank is one vLLM tensor-parallel rank
    (external launcher). Timed on the wall clock around `LLM.generate`, which returns after the
    device finished, max over ranks."""
    import tempfile

    import torch
    import torch.distributed as dist

    from furiosa_opt_models_b200.models import configs, synthetic

    cfg = configs.get(args.model)
    if cfg.get("weight_format", "bf16") != "bf16":
        if rank == 0:
            print(json.dumps({"impl": "vllm", "unavailable": "the vLLM arm serves the BF16 geometries"}))
        return
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    d = tempfile.mkdtemp(prefix="foa-vllm-")
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(synthetic.hf_config(cfg), f)
    total = args.input_len + args.output_len
    llm = LLM(model=d, load_format="dummy", skip_tokenizer_init=True, tensor_parallel_size=world,
              distributed_executor_backend="external_launcher" if world > 1 else None,
              max_model_len=total, max_num_seqs=args.concurrency, max_num_batched_tokens=8192,
              gpu_memory_utilization=0.8, enable_prefix_caching=False, seed=0, disable_log_stats=False)
    gen = torch.Generator().manual_seed(1234)
    prompts = [TokensPrompt(prompt_token_ids=torch.randint(0, cfg["vocab"], (args.input_len,), generator=gen).tolist())
               for _ in range(args.concurrency)]
    sp = SamplingParams(temperature=0.0, max_tokens=args.output_len, ignore_eos=True, detokenize=False)
    for _ in range(args.warmup):
        llm.generate(prompts, sp, use_tqdm=False)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    ttfts, tpots = [], []
    with sampler:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            outs = llm.generate(prompts, sp, use_tqdm=False)
            for o in outs:
                m = o.metrics
                if m is None:
                    continue
                ttfts.append(m.first_token_latency * 1e3)
                n = len(o.outputs[0].token_ids)
                if n > 1:
                    tpots.append((m.last_token_ts - m.first_token_ts) * 1e3 / (n - 1))
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    stats = torch.tensor([elapsed, statistics.median(ttfts) if ttfts else -1.0,
                          statistics.median(tpots) if tpots else -1.0], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    elapsed, ttft, tpot = stats.tolist()
    if rank == 0:
        value = args.steps * args.concurrency * args.output_len / elapsed
        print(json.dumps({
            "impl": "vllm", "metric": METRIC, "value": round(value, 1), "unit": "output tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(elapsed * 1e3 / args.steps, 3), "higher_is_better": True, "scaling": "strong",
            "dtype": "bf16", "data": "synthetic: uniform-random prompt token IDs; vLLM dummy weights",
            "p50_ttft_ms": round(ttft, 3), "p50_tpot_ms": round(tpot, 4),
            "config": {"model": f"{args.model} (shape of the named checkpoint)", "global_batch": args.concurrency,
                       "seq_len": total, "parallelism": f"tp{world}",
                       "stack": "stock vLLM (LLM.generate, its attention backend, CUDA graphs, its all-reduce)",
                       "timing": "wall clock around LLM.generate, max over ranks"},
            "clocks": sampler.summary(),
        }), flush=True)


def main() -> None:
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.impl == "vllm":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        if world > 1:
            import datetime

            import torch
            import torch.distributed as dist

            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device("cuda", local))
        vllm_arm(args, world, rank, local)
        return

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    if args.impl == "baseline":
        baseline_arm(args, torch, dist, world, rank, local)
        if world > 1:
            dist.destroy_process_group()
        return

    import furiosa_opt_engine as engine
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import configs
    from furiosa_opt_models_b200.parallel import tp as tp_mod

    cfg = configs.get(args.model)
    device = engine.Device(engine.Placement(list(range(world)), range(8)))
    model = engine._native._synthetic_decoder(device, cfg, tp=world, rank=rank, seed=0, std=0.02)
    if world > 1:
        tp_mod.attach(model, device)
    if args.no_graphs:
        model.set_graphs(False)
    total = args.input_len + args.output_len
    nblocks = args.concurrency * serving.blocks_for(total) + 16
    cache = engine.decoder.Cache(model.cache, nblocks)
    stream = torch.cuda.ExternalStream(device.stream)

    gen = torch.Generator().manual_seed(1234)
    prompts_host = [torch.randint(0, cfg["vocab"], (args.input_len,), generator=gen, dtype=torch.int32)
                    for _ in range(args.concurrency)]
    prompts = [engine.HostTensor.from_dlpack(p).to_hbm(device) for p in prompts_host]
    rows = min(model.rows, 8192)

    def new_wave():
        alloc = serving.BlockAllocator(nblocks)
        return [serving.Sequence(prompts[i], args.input_len, alloc.take(serving.blocks_for(total)))
                for i in range(args.concurrency)]

    def wave_device(record: bool):
        """One wave with device-resident tokens; CUDA events mark each call's end."""
        seqs = new_wave()
        marks = []
        start = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        ttft_marks = []
        for call in serving.prefill_calls(seqs, rows):
            serving.prefill(model, cache, seqs, call)
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            ttft_marks.append((ev, len(call)))
        for _ in range(args.output_len - 1):
            serving.decode(model, cache, seqs)
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            marks.append(ev)
        return start, ttft_marks, marks

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        wave_device(False)
    device.synchronize()
    launches_before = model.kernel_launches
    barrier()
    device.synchronize()
    sampler = ClockSampler(local)
    with sampler:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        waves = [wave_device(True) for _ in range(args.steps)]
        t1.record(stream)
        device.synchronize()
    barrier()
    launches = model.kernel_launches - launches_before
    ms = t0.elapsed_time(t1)
    ttfts, tpots = [], []
    for start, ttft_marks, marks in waves:
        for ev, n in ttft_marks:
            ttfts += [start.elapsed_time(ev)] * n
        prev = ttft_marks[-1][0]
        for ev in marks:
            tpots.append(prev.elapsed_time(ev))
            prev = ev
    stats = torch.tensor([ms, statistics.median(ttfts), statistics.median(tpots)], dtype=torch.float64,
                         device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms, ttft, tpot = stats.tolist()
    out_tokens = args.steps * args.concurrency * args.output_len
    value = out_tokens / (ms / 1000.0)

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, engine, serving, model, cache, device, prompts_host, nblocks, total, rows,
                      world, dist, barrier)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "output tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": {"fp8_block": "fp8 (W8A8, 128x128 block scales)", "nvfp4_a4": "nvfp4 (W4A4)",
                      "nvfp4": "nvfp4 weights, bf16 inputs (W4A16)"}.get(cfg.get("weight_format", "bf16"), "bf16"),
            "data": "synthetic: uniform-random prompt token IDs; random-init N(0,0.02) weights",
            "p50_ttft_ms": round(ttft, 3),
            "p50_tpot_ms": round(tpot, 4),
            "config": {
                "model": f"{args.model} (shape of the named checkpoint, "
                         f"{cfg.get('weight_format', 'bf16')} projections, BF16 KV cache)",
                "global_batch": args.concurrency,
                "seq_len": total,
                "input_len": args.input_len,
                "output_len": args.output_len,
                "parallelism": f"tp{world}",
                "l2": "inputs larger than L2: every step streams all weights (GBs) and the KV cache",
                "step": "one wave: prefill of every request, then output_len-1 greedy decode calls",
            },
            "clocks": sampler.summary(),
            "gpu_launches": int(launches),
            "e2e": e2e,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        tp_mod.detach(model)
        dist.destroy_process_group()


def run_e2e(args, engine, serving, model, cache, device, prompts_host, nblocks, total, rows, world,
            dist, barrier) -> dict:
    """The same waves end to end through the public API: prompts and every step's input tokens go
    host->device from pinned memory, every step's output tokens come back device->host."""
    import numpy as np
    from furiosa_opt_engine import decoder as dec

    # A host buffer holds every chip's bytes (a rank copies its own slice): the inputs replicated.
    pinned = [engine.HostBuffer(np.tile(p.numpy(), world)) for p in prompts_host]
    h2d = d2h = calls = 0

    def wave():
        nonlocal h2d, d2h, calls
        alloc = serving.BlockAllocator(nblocks)
        seqs = []
        for i in range(args.concurrency):
            buf = engine.HbmBuffer(device, args.input_len * 4)
            pinned[i].to_hbm(buf)
            h2d += args.input_len * 4
            t = engine.HbmTensor(buf, [args.input_len], "int32")
            seqs.append(serving.Sequence(t, args.input_len, alloc.take(serving.blocks_for(total))))
        last = np.zeros(args.concurrency, dtype=np.int32)
        for call in serving.prefill_calls(seqs, rows):
            out = serving.prefill(model, cache, seqs, call)
            h2d += model.last_staged_bytes
            host = out.to_host().numpy()
            d2h += host.nbytes
            calls += 1
            last[call] = host
        for _ in range(args.output_len - 1):
            step_in = engine.HostBuffer(np.tile(last, world))
            buf = engine.HbmBuffer(device, args.concurrency * 4)
            step_in.to_hbm(buf)
            h2d += args.concurrency * 4
            toks = engine.HbmTensor(buf, [args.concurrency], "int32")
            reqs = [dec.Request([s.blocks], s.cached, toks[k:k + 1], dec.Keep.LAST) for k, s in enumerate(seqs)]
            out = model.forward(reqs, cache)
            h2d += model.last_staged_bytes
            for s in seqs:
                s.cached += 1
            last = out.to_host().numpy()
            d2h += last.nbytes
            calls += 1

    wave()
    device.synchronize()
    h2d = d2h = calls = 0
    barrier()
    device.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        wave()
    device.synchronize()
    barrier()
    elapsed = time.perf_counter() - t0
    import torch

    t = torch.tensor([elapsed], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed = t.item()
    return {
        "value": round(args.steps * args.concurrency * args.output_len / elapsed, 1),
        "unit": "output tokens/s",
        "h2d_bytes_per_step": int(h2d / args.steps),
        "d2h_bytes_per_step": int(d2h / args.steps),
        "calls_per_step": int(calls / args.steps),
        "timing": "host wall clock between device syncs and a barrier, max over ranks",
    }


if __name__ == "__main__":
    main()
