"""Times one engine kernel on a named workload with CUDA events (and gives profilers a fixed launch
sequence: `--warmup` launches, then `--iters` timed ones, each after an L2 flush).

    python -m furiosa_opt_models_b200.utils.kernel_bench gemm --M 64 --N 4096 --K 4096 --format bf16
    python -m furiosa_opt_models_b200.utils.kernel_bench decode-attn --rows 64 --keys 2048
    python -m furiosa_opt_models_b200.utils.kernel_bench prefill-attn --rows 8192 --seqs 8
    python -m furiosa_opt_models_b200.utils.kernel_bench moe --tokens 64
    torchrun --nproc-per-node 2 -m furiosa_opt_models_b200.utils.kernel_bench tp-o-proj --rows 64

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
    """One GEMM shape. `--rotate R`: R distinct weight copies (together larger than L2) launched
    back to back without a flush, as a decoder's consecutive projections run; the per-launch time is
    the loop's. `--cta-trace`: per-CTA global-timer milestones of one launch in that loop."""
    from furiosa_opt_models_b200 import ops

    M, N, K = args.M, args.N, args.K
    a = torch.randn(M, K, device="cuda").bfloat16()
    fmt = args.format
    copies = max(1, args.rotate)
    ws = []
    for _ in range(copies):
        w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
        if fmt == "fp8":
            w = ops.quantize_fp8_block(w)
        elif fmt == "fp8_w8a16":
            import dataclasses

            w = dataclasses.replace(ops.quantize_fp8_block(w), format="fp8_block_w8a16")
        elif fmt == "nvfp4":
            w = ops.quantize_nvfp4(w)  # W4A16: BF16 inputs, E2M1 weights expanded on the fly
        elif fmt == "nvfp4a4":
            w = ops.nvfp4_w4a4(ops.quantize_nvfp4(w), float(a.float().abs().max()) / 2688)
        ws.append(w)
    wbytes = N * K * ({"fp8": 1 + 1 / 4096, "fp8_w8a16": 1 + 1 / 4096, "nvfp4": 0.5 + 1 / 16,
                       "nvfp4a4": 0.5 + 1 / 16}.get(fmt, 2))
    epi = {"bf16": ops.EPI_BF16, "f32": ops.EPI_F32, "swiglu": ops.EPI_SWIGLU}[args.epilogue]
    out = {}
    if copies == 1:
        us = _time(lambda: ops.gemm(a, ws[0], epilogue=epi, splits=args.splits, reduction=args.reduction,
                                    debug=args.debug, mode=args.mode),
                   args.warmup, args.iters)
    else:
        # Two traced launches in the middle of the loop: launch `mid` and the one after it.
        tr = torch.zeros(2, 8 * 1024, dtype=torch.int64, device="cuda")
        mid = copies // 2

        def loop(trace=False):
            for i, w in enumerate(ws):
                if args.impl == "cublas":
                    torch.matmul(a, w.t())  # the library reference point (BF16 only)
                    continue
                t = tr[i - mid] if trace and i in (mid, mid + 1) else None
                ops.gemm(a, w, epilogue=epi, splits=args.splits, cta_trace=t, reduction=args.reduction,
                         debug=args.debug, mode=args.mode)

        for _ in range(args.warmup):
            loop()
        torch.cuda.synchronize()
        run = loop
        if args.graph:
            # Captured once and replayed, as a decoder's calls run: no host work between launches.
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                loop()
                torch.cuda.synchronize()
                with torch.cuda.graph(g, stream=s):
                    loop(trace=args.cta_trace)
            torch.cuda.current_stream().wait_stream(s)
            run = g.replay
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            run()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / (args.iters * copies)
        if args.cta_trace and args.impl != "cublas":
            if not args.graph:
                loop(trace=True)
                torch.cuda.synchronize()
            both = tr.view(2, -1, 8).cpu().double()
            t0 = both[0][both[0][:, 0] > 0][:, 0].min()
            for j, name in ((0, "cta_us"), (1, "next_cta_us")):
                t = both[j][both[j][:, 0] > 0]
                rel = (t - t0) / 1000.0
                q = lambda col: [round(float(x), 2) for x in torch.quantile(rel[:, col], torch.tensor([0.0, 0.5, 1.0], dtype=torch.float64))]
                names = ["entry", "accumulator", "epilogue", "cluster_sync1", "pushed", "cluster_sync2", "reduced", "exit"]
                out[name] = {"ctas": int(t.shape[0])}
                out[name].update({n: q(c) for c, n in enumerate(names) if (t[:, c] > 0).all()})
    flops = 2 * M * N * K
    out.update(kernel="gemm", format=fmt, M=M, N=N, K=K, rotate=copies, us=round(us, 2),
               tflops=round(flops / us / 1e6, 1), weight_gbs=round(wbytes / us / 1e3, 1))
    return out


def decode_attn(args) -> dict:
    from furiosa_opt_models_b200 import ops

    rows, keys, qh, kvh, d = args.rows, args.keys, args.q_heads, args.kv_heads, 128
    nb = (keys + 15) // 16
    cache = torch.randn(rows * nb, 2, kvh, 16, d, device="cuda").bfloat16()
    table = torch.arange(rows * nb, dtype=torch.int32, device="cuda")
    seg = torch.tensor([[r, 1, keys - 1, r * nb, nb] for r in range(rows)], dtype=torch.int32, device="cuda")
    q = torch.randn(rows, qh, d, device="cuda").bfloat16()
    us = _time(lambda: ops.paged_decode(q, cache, table, seg, kvh, keys, keys_per_split=args.split,
                                        warps=args.warps, stages=args.stages),
               args.warmup, args.iters)
    kv_bytes = rows * keys * kvh * d * 2 * 2
    return dict(kernel="paged_decode", rows=rows, keys=keys, kv_heads=kvh, split=args.split, us=round(us, 2),
                kv_gbs=round(kv_bytes / us / 1e3, 1))


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
    us = _time(lambda: ops.paged_prefill(q, cache, table, seg, kvh, work, tensor_cores=not args.mma_sync),
               args.warmup, args.iters)
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


def tp_o_proj(args) -> dict:
    """Layer 0's attention output projection under tensor parallelism, device-timed on every rank
    (the maximum reported): the GEMM writing its FP32 partial locally, the scatter kernel storing it
    over NVLink into the reducing ranks' receive slots and the rank-ordered reducer + residual +
    RMSNorm polling for it ("fused"); the GEMM alone ("local"); the scatter and reducer alone on a
    partial already in place ("collective")."""
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
    # Layer 0 alone, BF16 weights: the projection's geometry is the model's.
    cfg = configs.get(args.model, layers=1, weight_format="bf16")
    device = engine.Device(engine.Placement(list(range(world)), range(8)))
    model = _native._synthetic_decoder(device, cfg, tp=world, rank=rank, seed=0, std=0.02)
    tp.attach(model, device)
    H, D = cfg["hidden"], cfg.get("head_dim", 128)
    K = cfg["q_heads"] // world * D
    a = torch.randn(args.rows, K, device="cuda").bfloat16()
    r = _native._tp_bench_o_proj(model, args.rows, a.data_ptr(), args.iters)
    t = torch.tensor([r["fused"], r["local"], r["split_gemm"], r["split_norm"], r["collective"]],
                     dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    fused_us, local_us, coll_us = t[0].item() * 1000.0, t[1].item() * 1000.0, t[4].item() * 1000.0
    split = {"gemm_us": round(t[2].item() * 1000.0, 2), "scatter_reduce_norm_us": round(t[3].item() * 1000.0, 2)}
    tp.detach(model)
    dist.destroy_process_group()
    one_shot = r["two_shot"] == 0
    # Bytes each rank must move across NVLink: FP32 partials stored into the peers (every row, or
    # each peer's slice), plus (two-shot) its slice's BF16 normed rows stored into every peer.
    nvlink = (args.rows * H * 4 * (world - 1) if one_shot
              else args.rows * H * 4 * (world - 1) / world + args.rows * H * 2 * (world - 1) / world)
    peaks = _peaks()
    roof = {"nvlink_us": nvlink / 770e3,
            "weights_us": H * K * 2 / (peaks["hbm_gbs"] * 1e3),
            "compute_us": 2 * args.rows * H * K / (peaks["bf16_tflops"] * 1e6)}
    bound = max(roof.values())
    return dict(kernel="tp_o_proj_add_norm", world=world, rows=args.rows, hidden=H, K=K,
                mode="one-shot" if one_shot else "two-shot", fused_us=round(fused_us, 2),
                local_gemm_us=round(local_us, 2), collective_us=round(coll_us, 2),
                overlap_us=round(local_us + coll_us - fused_us, 2),
                events_between_kernels=split,
                trace_local_us=[round(r[f"trace_local_{i}"], 2) for i in range(8)],
                trace_fused_us=[round(r[f"trace_fused_{i}"], 2) for i in range(11)],
                nvlink_bytes_per_rank=int(nvlink), roofline_us={k: round(v, 2) for k, v in roof.items()},
                roofline_fraction=round(bound / fused_us, 3), _rank=rank)


def _peaks() -> dict:
    import os

    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"])}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = p.add_subparsers(dest="what", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--M", type=int, default=64)
    g.add_argument("--N", type=int, default=4096)
    g.add_argument("--K", type=int, default=4096)
    g.add_argument("--format", default="bf16", choices=["bf16", "fp8", "fp8_w8a16", "nvfp4", "nvfp4a4"])
    g.add_argument("--epilogue", default="bf16", choices=["bf16", "f32", "swiglu"])
    g.add_argument("--splits", type=int, default=0)
    g.add_argument("--rotate", type=int, default=1)
    g.add_argument("--cta-trace", action="store_true")
    g.add_argument("--graph", action="store_true")
    g.add_argument("--impl", default="engine", choices=["engine", "cublas"])
    g.add_argument("--mode", type=int, default=0, choices=[0, 1, 2],
                   help="0: the plan's choice (CUDA-core weight stream up to 8 rows), 1: rows mapping, 2: swap mapping")
    g.add_argument("--debug", type=int, default=0, choices=[0, 1, 2, 3],
                   help="leave out the output stores (1), the accumulator reads (2) or both (measurement)")
    g.add_argument("--reduction", type=int, default=0, choices=[0, 1, 2],
                   help="split-K partials meet by the plan's choice (0), global scratch (1) or the cluster (2)")
    d = sub.add_parser("decode-attn")
    d.add_argument("--rows", type=int, default=64)
    d.add_argument("--keys", type=int, default=2048)
    d.add_argument("--q-heads", type=int, default=16)
    d.add_argument("--kv-heads", type=int, default=8)
    d.add_argument("--split", type=int, default=2048, help="keys per split")
    d.add_argument("--warps", type=int, default=0, help="warps a CTA (2-4; 0 the engine's default)")
    d.add_argument("--stages", type=int, default=0, help="16-key blocks in flight a warp (2-3; 0 default)")
    f = sub.add_parser("prefill-attn")
    f.add_argument("--rows", type=int, default=8192)
    f.add_argument("--seqs", type=int, default=8)
    f.add_argument("--q-heads", type=int, default=16)
    f.add_argument("--kv-heads", type=int, default=8)
    f.add_argument("--mma-sync", action="store_true", help="the mma.sync kernel instead of tcgen05")
    m = sub.add_parser("moe")
    m.add_argument("--tokens", type=int, default=64)
    a = sub.add_parser("tp-o-proj")
    a.add_argument("--rows", type=int, default=64)
    a.add_argument("--model", default="qwen3-1.7b")
    for s in (g, d, f, m, a):
        s.add_argument("--warmup", type=int, default=3)
        s.add_argument("--iters", type=int, default=10)
    args = p.parse_args()
    out = {"gemm": gemm, "decode-attn": decode_attn, "prefill-attn": prefill_attn, "moe": moe,
           "tp-o-proj": tp_o_proj}[args.what](args)
    if out.pop("_rank", 0) == 0:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
