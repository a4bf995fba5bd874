"""Times one engine kernel on a named workload with CUDA events (and gives profilers a fixed launch
sequence: `--warmup` launches, then `--iters` timed ones, each after an L2 flush).

    python -m furiosa_opt_models_b200.utils.kernel_bench gemm --M 64 --N 4096 --K 4096 --format bf16
    python -m furiosa_opt_models_b200.utils.kernel_bench decode-attn --rows 64 --keys 2048
    python -m furiosa_opt_models_b200.utils.kernel_bench prefill-attn --rows 8192 --seqs 8
    python -m furiosa_opt_models_b200.utils.kernel_bench moe --tokens 64
    torchrun --nproc-per-node 2 -m furiosa_opt_models_b200.utils.kernel_bench add-norm --rows 64

Prints one JSON line: the mean device time per launch and the algorithmic bytes and FLOPs.
"""

from __future__ import annotations

import argparse
import json

import torch


def _time(fn, warmup: int, iters: int) -> float:
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        total += a.elapsed_time(b)
    return total / max(iters, 1) * 1000.0  # microseconds


def gemm(args) -> dict:
    from furiosa_opt_models_b200 import ops

    M, N, K = args.M, args.N, args.K
    a = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    fmt = args.format
    if fmt == "fp8":
        w = ops.quantize_fp8_block(w)
        wbytes = N * K * (1 + 1 / 4096)
    elif fmt == "nvfp4a4":
        w = ops.nvfp4_w4a4(ops.quantize_nvfp4(w), float(a.float().abs().max()) / 2688)
        wbytes = N * K * (0.5 + 1 / 16)
    else:
        wbytes = N * K * 2
    epi = {"bf16": ops.EPI_BF16, "f32": ops.EPI_F32, "swiglu": ops.EPI_SWIGLU}[args.epilogue]
    us = _time(lambda: ops.gemm(a, w, epilogue=epi), args.warmup, args.iters)
    flops = 2 * M * N * K
    return dict(kernel="gemm", format=fmt, M=M, N=N, K=K, us=round(us, 2), tflops=round(flops / us / 1e6, 1),
                weight_gbs=round(wbytes / us / 1e3, 1))


def decode_attn(args) -> dict:
    from furiosa_opt_models_b200 import ops

    rows, keys, qh, kvh, d = args.rows, args.keys, args.q_heads, args.kv_heads, 128
    nb = (keys + 15) // 16
    cache = torch.randn(rows * nb, 2, kvh, 16, d, device="cuda").bfloat16()
    table = torch.arange(rows * nb, dtype=torch.int32, device="cuda")
    seg = torch.tensor([[r, 1, keys - 1, r * nb, nb] for r in range(rows)], dtype=torch.int32, device="cuda")
    q = torch.randn(rows, qh, d, device="cuda").bfloat16()
    us = _time(lambda: ops.paged_decode(q, cache, table, seg, kvh, keys), args.warmup, args.iters)
    kv_bytes = rows * keys * kvh * d * 2 * 2
    return dict(kernel="paged_decode", rows=rows, keys=keys, us=round(us, 2), kv_gbs=round(kv_bytes / us / 1e3, 1))


def prefill_attn(args) -> dict:
    from furiosa_opt_models_b200 import ops

    seqs, per, qh, kvh, d = args.seqs, args.rows // args.seqs, args.q_heads, args.kv_heads, 128
    nb = (per + 15) // 16
    cache = torch.randn(seqs * nb, 2, kvh, 16, d, device="cuda").bfloat16()
    table = torch.arange(seqs * nb, dtype=torch.int32, device="cuda")
    seg_cpu = torch.tensor([[s * per, per, 0, s * nb, nb] for s in range(seqs)], dtype=torch.int32)
    seg = seg_cpu.cuda()
    work = ops.prefill_work(seg_cpu, qh // kvh).cuda()
    q = torch.randn(seqs * per, qh, d, device="cuda").bfloat16()
    us = _time(lambda: ops.paged_prefill(q, cache, table, seg, kvh, work), args.warmup, args.iters)
    flops = seqs * 2 * 2 * qh * d * per * per / 2  # causal: QK and PV over half the square
    return dict(kernel="paged_prefill", rows=seqs * per, seqs=seqs, us=round(us, 2), tflops=round(flops / us / 1e6, 1))


def moe(args) -> dict:
    from furiosa_opt_models_b200 import ops

    T, H, I, E, k = args.tokens, 2048, 768, 128, 8
    h = torch.randn(T, H, device="cuda").bfloat16()
    router = (torch.randn(E, H, device="cuda") * 0.02).bfloat16()
    gate_up = (torch.randn(E, 2 * I, H, device="cuda") * 0.02).bfloat16()
    down = (torch.randn(E, H, I, device="cuda") * 0.02).bfloat16()
    per = T * k / E
    tile = 16 if per <= 16 else 32 if per <= 32 else 64 if per <= 64 else 128

    def block():
        logits = ops.gemm(h, router)
        ids, w = ops.moe_route(logits, k, True)
        pos, src, tile_expert, tiles = ops.moe_align(ids, E, tile)
        xs = ops.moe_gather(h, src, tiles, tile)
        act = ops.grouped_gemm(xs, gate_up, tiles, tile_expert, tile, epilogue=ops.EPI_SWIGLU)
        y = ops.grouped_gemm(act, down, tiles, tile_expert, tile)
        return ops.moe_combine(y, pos, w, h.clone())

    us = _time(block, args.warmup, args.iters)
    touched = min(E, T * k)
    wbytes = touched * (2 * I * H + H * I) * 2
    return dict(kernel="moe_block", tokens=T, tile=tile, us=round(us, 2), expert_weight_gbs=round(wbytes / us / 1e3, 1))


def add_norm(args) -> dict:
    """The fused tensor-parallel add+norm (rank-ordered FP32 sum over NVLink + residual +
    RMSNorm), device-timed on every rank, the maximum reported."""
    import datetime
    import os

    import torch.distributed as dist

    import furiosa_opt_engine as engine
    from furiosa_opt_engine import _native
    from furiosa_opt_models_b200.models import configs
    from furiosa_opt_models_b200.parallel import tp

    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    cfg = configs.get(args.model)
    device = engine.Device(engine.Placement(list(range(world)), range(8)))
    model = _native._synthetic_decoder(device, cfg, tp=world, rank=rank, seed=0, std=0.02)
    tp.attach(model, device)
    ms = _native._tp_bench_add_norm(model, args.rows, args.iters)
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = t.item() * 1000.0
    H = cfg["hidden"]
    one_shot = args.rows * H * 4 * (world - 1) <= (1 << 20) or args.rows < world
    nvlink = (args.rows * H * 4 * (world - 1) if one_shot
              else args.rows * H * 4 * (world - 1) / world + 2 * args.rows * H * 2 * (world - 1) / world)
    tp.detach(model)
    dist.destroy_process_group()
    return dict(kernel="tp_add_norm", world=world, rows=args.rows, hidden=H, mode="one-shot" if one_shot else "two-shot",
                us=round(us, 2), nvlink_bytes_per_rank=int(nvlink),
                nvlink_gbs=round(nvlink / us / 1e3, 1), roofline_fraction_of_770=round(nvlink / us / 1e3 / 770, 3),
                _rank=rank)


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = p.add_subparsers(dest="what", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--M", type=int, default=64)
    g.add_argument("--N", type=int, default=4096)
    g.add_argument("--K", type=int, default=4096)
    g.add_argument("--format", default="bf16", choices=["bf16", "fp8", "nvfp4a4"])
    g.add_argument("--epilogue", default="bf16", choices=["bf16", "f32", "swiglu"])
    d = sub.add_parser("decode-attn")
    d.add_argument("--rows", type=int, default=64)
    d.add_argument("--keys", type=int, default=2048)
    d.add_argument("--q-heads", type=int, default=16)
    d.add_argument("--kv-heads", type=int, default=8)
    f = sub.add_parser("prefill-attn")
    f.add_argument("--rows", type=int, default=8192)
    f.add_argument("--seqs", type=int, default=8)
    f.add_argument("--q-heads", type=int, default=16)
    f.add_argument("--kv-heads", type=int, default=8)
    m = sub.add_parser("moe")
    m.add_argument("--tokens", type=int, default=64)
    a = sub.add_parser("add-norm")
    a.add_argument("--rows", type=int, default=64)
    a.add_argument("--model", default="qwen3-1.7b")
    for s in (g, d, f, m, a):
        s.add_argument("--warmup", type=int, default=3)
        s.add_argument("--iters", type=int, default=10)
    args = p.parse_args()
    out = {"gemm": gemm, "decode-attn": decode_attn, "prefill-attn": prefill_attn, "moe": moe,
           "add-norm": add_norm}[args.what](args)
    if out.pop("_rank", 0) == 0:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
