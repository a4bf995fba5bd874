"""The forward benchmark's cases and the metric records made from traces and serving summaries
(the reference's .github/actions/metrics/action.yml and crates/furiosa-opt-engine/tests/forward.rs)."""

import json

import pytest

from furiosa_opt_models_b200.bench import forward, inventory, metrics


def test_cases_of_the_nightly_workloads():
    lengths, widths = forward.workloads(inventory(), "nightly")
    assert lengths == [(1024, 1024), (1024, 8192), (8192, 1024)]
    assert widths == [16]  # the concurrencies every nightly workload runs
    cases = forward.cases(lengths, widths, chunk=1024, window=40960)
    names = [c[0] for c in cases]
    assert names == sorted(names)
    # One prefill case per input length: the last chunk of the prompt.
    assert ("in-8192-prefill-chunk-1024", 7168, 1024, 1) in cases
    assert ("in-1024-prefill-chunk-1024", 0, 1024, 1) in cases
    assert names.count("in-1024-prefill-chunk-1024") == 1
    # Decode halfway through the output, for one request and each common concurrency.
    assert ("in-1024-out-8192-decode-rows-16", 1024 + 4096, 1, 16) in cases
    assert ("in-8192-out-1024-decode-rows-1", 8192 + 512, 1, 1) in cases
    assert len(cases) == 2 + 3 * 2


def test_cases_past_the_window_or_the_rows_are_not_measured():
    cases = forward.cases([(8192, 1024)], [1, 4, 16], chunk=4, window=8192)
    names = {c[0] for c in cases}
    assert names == {"in-8192-prefill-chunk-4"}  # decode at 8704 positions is past the window
    cases = forward.cases([(128, 128)], [16], chunk=8, window=4096)
    assert {c[0] for c in cases} == {"in-128-prefill-chunk-8", "in-128-out-128-decode-rows-1"}


def test_trace_directory_and_model_tag():
    d = forward.trace_dir("trace", "Qwen/Qwen3-1.7B")
    assert d.endswith("qwen--qwen3-1.7b")
    assert metrics.model_tag(d) == "qwen/qwen3-1.7b"
    assert forward.hub_id(inventory(), "qwen3-1.7b") == "Qwen/Qwen3-1.7B"
    assert forward.hub_id(inventory(), "tiny-qwen3") == "synthetic/tiny-qwen3"


def _span(name, cat, ts, dur, **args):
    e = {"name": name, "cat": cat, "ph": "X", "ts": ts, "dur": dur, "pid": 1, "tid": 0}
    if args:
        e["args"] = args
    return e


def test_trace_records(tmp_path):
    events = []
    # Three measured calls of one case, two of another; kernel spans land inside their calls.
    for step, (t, total) in enumerate([(0, 900.0), (1000, 1100.0), (3000, 1000.0)], start=1):
        events.append(_span("forward", "bench", t, total, case="in-16-decode", step=step))
        events.append(_span("forward", "call", t + 1, 20.0))  # the engine's own host span
        events.append(_span("forward.device", "GPU", t + 30, total - 50, ns=0))
        events.append(_span("gemm", "GPU", t + 40, 10.0, ns=10_000 * step))
        events.append(_span("gemm", "GPU", t + 60, 10.0, ns=5_000))
        events.append(_span("paged_decode", "GPU", t + 80, 3.0, ns=3_000))
    events.append(_span("forward", "bench", 10_000, 2000.0, case="in-16-prefill", step=1))
    events.append(_span("forward", "bench", 13_000, 4000.0, case="in-16-prefill", step=2))
    events.append(_span("gemm", "GPU", 9_000, 5.0, ns=1))  # before every call: ignored
    events.append(_span("request", "framework", 0, 5000.0))
    events.append(_span("request", "framework", 0, 7000.0))
    d = tmp_path / "trace" / "qwen--qwen3-1.7b"
    d.mkdir(parents=True)
    (d / "forward.json").write_text(json.dumps({"traceEvents": events}))
    recs = metrics.collect(str(tmp_path / "trace"), None)
    by = {(r["metric"], tuple(r["tags"])): r["value"] for r in recs}
    base = ("model:qwen/qwen3-1.7b", "test:forward")
    assert by[("furiosa_opt.forward.step_ms", base + ("case:in-16-decode",))] == pytest.approx(1.0)
    assert by[("furiosa_opt.forward.step_ms", base + ("case:in-16-prefill",))] == pytest.approx(2.0)
    assert by[("furiosa_opt.forward.device_ms", base + ("case:in-16-decode",))] == pytest.approx(0.95)
    # A kernel's time in a call sums its launches; the value is the median over calls.
    assert by[("furiosa_opt.kernel.ns", base + ("case:in-16-decode", "kernel:gemm"))] == pytest.approx(25_000)
    assert by[("furiosa_opt.kernel.ns", base + ("case:in-16-decode", "kernel:paged_decode"))] == 3_000
    assert by[("furiosa_opt.serving.request_ms", base)] == pytest.approx(5.0)
    assert not any("case:in-16-prefill" in r["tags"] and r["metric"] == "furiosa_opt.kernel.ns" for r in recs)


def test_summary_records(tmp_path):
    d = tmp_path / "sweep" / "qwen--qwen3-1.7b" / "in-1024-out-1024" / "16"
    d.mkdir(parents=True)
    (d / "summary.json").write_text(json.dumps({
        "completed": 32, "num_prompts": 32, "failed": 0, "max_concurrency": 16,
        "median_ttft_ms": 41.5, "median_tpot_ms": 3.25, "median_e2el_ms": 3400.0}))
    recs = metrics.collect(None, str(tmp_path / "sweep"))
    tags = ["model:qwen/qwen3-1.7b", "batch:16", "scenario:in-1024-out-1024"]
    assert recs == [
        {"metric": "furiosa_opt.serving.ttft_ms", "tags": tags, "value": 41.5},
        {"metric": "furiosa_opt.serving.tpot_ms", "tags": tags, "value": 3.25},
        {"metric": "furiosa_opt.serving.request_ms", "tags": tags, "value": 3400.0},
    ]
    (d / "summary.json").write_text(json.dumps({"completed": 31, "num_prompts": 32}))
    with pytest.raises(metrics.IncompleteMeasurements):
        metrics.collect(None, str(tmp_path / "sweep"))


def test_tags_are_normalized():
    assert metrics.tag("Qwen/Qwen3 1.7B:x") == "qwen/qwen3_1.7b_x"


def test_host_span_args_reach_the_trace(tmp_path):
    from furiosa_opt_engine import _native

    _native._trace_flush("/dev/null")
    t0 = _native._trace_now_ns()
    _native._trace_span("forward", "bench", t0, t0 + 1000, json.dumps({"case": "c", "step": 3}))
    path = _native._trace_flush(str(tmp_path / "t.json"))
    (e,) = json.load(open(path))["traceEvents"]
    assert e["args"] == {"case": "c", "step": 3}
    with pytest.raises(ValueError, match="args is a JSON object"):
        _native._trace_span("x", "y", t0, t0 + 1, "[1]")
