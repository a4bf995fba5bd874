"""Metric records (JSON lines) from forward-benchmark traces and serving summaries.

Records are `{"metric": ..., "tags": [...], "value": ...}`, one per line, each value a median:

- `furiosa_opt.forward.step_ms` (tags model, test, case): a measured call's `forward` span, from
  submission to the device's completion;
- `furiosa_opt.forward.device_ms` (same tags): the engine's device span of that call;
- `furiosa_opt.kernel.ns` (tags model, test, case, kernel): a kernel's device time in one call,
  summed over its launches in the call (traces taken under FURIOSA_OPT_PROFILE=trace);
- `furiosa_opt.serving.request_ms` (tags model, test): whole `request` spans a framework recorded;
- `furiosa_opt.serving.{ttft,tpot,request}_ms` (tags model, batch, scenario): the medians of a
  `vllm bench serve` summary.

A trace lives at `<traces>/<org>--<name>/<test>.json`, a summary at
`<sweep>/<org>--<name>/<lengths>/<widths>/summary.json`; the model tag is `<org>/<name>`. Tag values
are lowercased with characters outside `[a-z0-9_./-]` replaced by `_`.

Reference: .github/actions/metrics/action.yml:10-90 (the same records from the reference's
traces, which time kernels in device cycles; here kernels are timed in nanoseconds by CUDA events).

    python -m furiosa_opt_models_b200.bench.metrics [--traces trace] [--sweep sweep] > metrics.jsonl
"""

from __future__ import annotations

import argparse
import bisect
import glob
import json
import os
import re
import sys
from collections import defaultdict


class IncompleteMeasurements(ValueError):
    pass


def tag(value) -> str:
    return re.sub(r"[^a-z0-9_./-]", "_", str(value).lower())


def median(values: list[float]) -> float:
    s = sorted(values)
    return s[(len(s) - 1) // 2]


def model_tag(directory: str) -> str:
    org, _, name = os.path.basename(os.path.normpath(directory)).partition("--")
    return f"{org}/{name}" if name else org


def steps(events: list[dict]) -> list[dict]:
    """Each measured call (a `forward` span with a `case`) with the engine's spans inside it."""
    out = []
    for e in events:
        args = e.get("args") or {}
        if e.get("name") == "forward" and e.get("ph") == "X" and "case" in args:
            out.append({"case": args["case"], "step": args.get("step"), "begin": float(e["ts"]),
                        "end": float(e["ts"]) + float(e["dur"]), "device": [], "kernels": []})
    out.sort(key=lambda s: s["begin"])
    if not out:
        return out
    begins = [s["begin"] for s in out]
    for e in events:
        if e.get("cat") != "GPU" or e.get("ph") != "X":
            continue
        ts, dur = float(e["ts"]), float(e["dur"])
        # Calls run one at a time: a device span belongs to the call whose window holds its start
        # (its end may lie a little past the window, by the host-device clock alignment).
        i = bisect.bisect_right(begins, ts) - 1
        if i < 0 or ts > out[i]["end"]:
            continue
        s = out[i]
        if e.get("name") == "forward.device":
            s["device"].append(dur / 1000.0)
        else:
            ns = (e.get("args") or {}).get("ns", dur * 1000.0)
            s["kernels"].append((e["name"], float(ns)))
    return out


def validate(step: dict) -> dict:
    if step["end"] < step["begin"]:
        raise IncompleteMeasurements(f"case {step['case']}: a call ends before it begins")
    if any(ns < 0 for _, ns in step["kernels"]):
        raise IncompleteMeasurements(f"case {step['case']}: a kernel span ends before it begins")
    return step


def trace_records(path: str, model: str, test: str) -> list[dict]:
    with open(path) as f:
        doc = json.load(f)
    events = doc["traceEvents"] if isinstance(doc, dict) else doc
    samples: dict[tuple, list[float]] = defaultdict(list)
    for s in map(validate, steps(events)):
        samples[("forward.step_ms", s["case"], None)].append((s["end"] - s["begin"]) / 1000.0)
        if s["device"]:
            samples[("forward.device_ms", s["case"], None)].append(sum(s["device"]))
        per_kernel: dict[str, float] = defaultdict(float)
        for name, ns in s["kernels"]:
            per_kernel[tag(name)] += ns
        for name, ns in per_kernel.items():
            samples[("kernel.ns", s["case"], name)].append(ns)
    out = []
    for (metric, case, kernel), values in sorted(samples.items(), key=lambda kv: (kv[0][0], kv[0][1], kv[0][2] or "")):
        tags = [f"model:{tag(model)}", f"test:{tag(test)}", f"case:{tag(case)}"]
        if kernel is not None:
            tags.append(f"kernel:{kernel}")
        out.append({"metric": f"furiosa_opt.{metric}", "tags": tags, "value": median(values)})
    requests = [float(e["dur"]) / 1000.0 for e in events if e.get("name") == "request" and e.get("ph") == "X"]
    if requests:
        out.append({"metric": "furiosa_opt.serving.request_ms",
                    "tags": [f"model:{tag(model)}", f"test:{tag(test)}"], "value": median(requests)})
    return out


def summary_records(path: str, model: str, scenario: str) -> list[dict]:
    with open(path) as f:
        doc = json.load(f)
    out = []
    for s in doc if isinstance(doc, list) else [doc]:
        if s.get("completed") != s.get("num_prompts") or (s.get("failed") or 0) != 0:
            raise IncompleteMeasurements(f"{path}: incomplete serving measurements")
        for metric, field in (("ttft", "ttft"), ("tpot", "tpot"), ("request", "e2el")):
            value = s.get(f"median_{field}_ms")
            if value is None:
                continue
            out.append({"metric": f"furiosa_opt.serving.{metric}_ms",
                        "tags": [f"model:{tag(model)}", f"batch:{tag(s.get('max_concurrency'))}",
                                 f"scenario:{tag(scenario)}"],
                        "value": value})
    return out


def collect(traces: str | None, sweep: str | None) -> list[dict]:
    out = []
    if traces:
        for path in sorted(glob.glob(os.path.join(traces, "*", "*.json"))):
            d = os.path.dirname(path)
            out += trace_records(path, model_tag(d), os.path.splitext(os.path.basename(path))[0])
    if sweep:
        for path in sorted(glob.glob(os.path.join(sweep, "*", "*", "*", "summary.json"))):
            scenario_dir = os.path.dirname(os.path.dirname(path))
            out += summary_records(path, model_tag(os.path.dirname(scenario_dir)), os.path.basename(scenario_dir))
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--traces", default="trace")
    p.add_argument("--sweep", default="sweep")
    a = p.parse_args(argv)
    for r in collect(a.traces, a.sweep):
        print(json.dumps(r))
    return 0


if __name__ == "__main__":
    sys.exit(main())
