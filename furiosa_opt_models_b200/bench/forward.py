"""Forward-phase benchmark: the calls each serving workload reaches, timed one at a time.

For every text workload (input, output) of the inventory's tier, the cases are:

- `in-{input}-prefill-chunk-{chunk}`: a prompt's last chunk, `chunk` rows appended after
  `input - chunk` cached positions, one request (`chunk` is the decoder's rows per call, at most
  the prompt);
- `in-{input}-out-{output}-decode-rows-{rows}`: a decode step halfway through the output, one row
  appended after `input + output / 2` cached positions, for one request and for each concurrency
  that every workload of the tier runs.

A case past the decoder's window, or with more requests than a call takes rows, is not measured.
Each case runs `warmups` unmeasured calls, then `repetitions` measured ones. A measured call is a
`forward` span (args `case`, `step`) from the call's submission to the device's completion; the
spans go to `<out>/<org>--<name>/forward.json` together with the engine's own spans (its device
span per call, and a span per kernel under FURIOSA_OPT_PROFILE=trace), and
`furiosa_opt_models_b200.bench.metrics` reads step and kernel times from that file. The timed calls
attend to cache pages that were never filled: timing does not depend on their values. The weights are random (N(0, 0.02)) in the shape
of the named model.

Reference: crates/furiosa-opt-engine/tests/forward.rs:47-160 (cases, warm-ups, repetitions and
the span per measured call), :162-195 (workloads from the inventory), .github/benchmarks.json.

    python -m furiosa_opt_models_b200.bench.forward --model qwen3-1.7b [--out trace] [--tier nightly]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys

from . import inventory


def workloads(inv: dict, tier: str = "nightly") -> tuple[list[tuple[int, int]], list[int]]:
    """The tier's (input, output) lengths and the concurrencies that every one of them runs."""
    tasks = inv["text"][tier]
    lengths = [(int(w["input"]), int(w["output"])) for w in tasks]
    common = [int(x) for x in tasks[0]["widths"] if all(x in w["widths"] for w in tasks)]
    return lengths, common


def cases(lengths: list[tuple[int, int]], widths: list[int], chunk: int,
          window: int) -> list[tuple[str, int, int, int]]:
    """Each case as (name, cached positions, tokens a request appends, requests), sorted by name;
    workloads of one input length share their prefill case."""
    out = set()
    for inp, outp in lengths:
        c = min(chunk, inp)
        out.add((f"in-{inp}-prefill-chunk-{c}", inp - c, c, 1))
        for rows in [1, *widths]:
            out.add((f"in-{inp}-out-{outp}-decode-rows-{rows}", inp + outp // 2, 1, rows))
    keep = [k for k in out if k[1] + k[2] <= window and k[3] <= chunk]
    return sorted(keep)


def trace_dir(root: str, hub_id: str) -> str:
    """`<root>/<org>--<name>` of a hub ID, lowercase."""
    return os.path.join(root, hub_id.lower().replace("/", "--"))


def hub_id(inv: dict, model: str) -> str:
    for m in inv.get("models", []):
        if m.get("config") == model:
            return m["id"]
    return f"synthetic/{model}"


def parse(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", default="qwen3-1.7b", help="a configuration of furiosa_opt_models_b200.models.configs")
    p.add_argument("--id", default=None, help="hub ID that names the trace directory (default: the inventory's)")
    p.add_argument("--out", default="trace")
    p.add_argument("--tier", default="nightly", choices=["nightly", "gate"])
    p.add_argument("--warmups", type=int, default=None)
    p.add_argument("--repetitions", type=int, default=None)
    p.add_argument("--max-input", type=int, default=None, help="skip workloads with longer prompts")
    p.add_argument("--profile", default=None, choices=["info", "debug", "trace"],
                   help="engine trace level (default: FURIOSA_OPT_PROFILE, else info)")
    return p.parse_args(argv)


def main(argv=None) -> int:
    args = parse(argv)
    inv = inventory()
    warmups = args.warmups if args.warmups is not None else inv["forward"]["warmups"]
    reps = args.repetitions if args.repetitions is not None else inv["forward"]["repetitions"]
    if reps < 1:
        raise SystemExit("--repetitions must be at least 1")

    import torch

    import furiosa_opt_engine as engine
    from furiosa_opt_engine import _native
    from furiosa_opt_engine import decoder as dec
    from furiosa_opt_models_b200.models import configs

    if args.profile:
        _native._trace_set_level(args.profile)
    elif _native._trace_level() == "off":
        _native._trace_set_level("info")

    cfg = configs.get(args.model)
    device = engine.Device(engine.Placement([0], range(8)))
    model = _native._synthetic_decoder(device, cfg, tp=1, rank=0, seed=0, std=0.02)
    spec = model.cache
    window = model.window  # positions a sequence reaches at most
    block = spec.pools[spec.groups[0].pool].block
    lengths, widths = workloads(inv, args.tier)
    if args.max_input is not None:
        lengths = [(i, o) for i, o in lengths if i <= args.max_input]
    todo = cases(lengths, widths, model.rows, window)
    if not todo:
        raise SystemExit("no case of the workloads fits this decoder")

    used = lambda cached, tokens: -(-(cached + tokens) // block)  # noqa: E731
    blocks = max(used(c, t) for _, c, t, _ in todo)
    rows = max(r for *_, r in todo)
    cache = dec.Cache(spec, blocks * rows)
    ids = engine.HostTensor.from_dlpack(
        torch.zeros(max(t * r for _, _, t, r in todo), dtype=torch.int32)).to_hbm(device)

    out_dir = trace_dir(args.out, args.id or hub_id(inv, args.model))
    os.makedirs(out_dir, exist_ok=True)
    summary = []
    for name, cached, tokens, count in todo:
        reqs = [dec.Request([list(range(r * blocks, r * blocks + used(cached, tokens)))], cached,
                            ids[r * tokens:(r + 1) * tokens], dec.Keep.LAST) for r in range(count)]
        times = []
        for sample in range(warmups + reps):
            t0 = _native._trace_now_ns()
            model.forward(reqs, cache)
            device.synchronize()
            t1 = _native._trace_now_ns()
            if sample >= warmups:
                step = sample - warmups + 1
                _native._trace_span("forward", "bench", t0, t1, json.dumps({"case": name, "step": step}))
                times.append((t1 - t0) / 1e6)
        line = {"case": name, "cached": cached, "tokens": tokens, "requests": count,
                "median_ms": round(statistics.median(times), 4)}
        summary.append(line)
        print(json.dumps(line), flush=True)
    path = _native._trace_flush(os.path.join(out_dir, "forward.json"))
    print(json.dumps({"trace": path, "model": args.model, "cases": len(summary)}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
