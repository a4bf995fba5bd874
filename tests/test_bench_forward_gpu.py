"""The forward benchmark on the GPU: every case of the gate workload is measured, and the metric
records read its step, device and kernel times back from the trace."""

import json

import pytest

pytestmark = pytest.mark.gpu


def test_forward_benchmark_trace_gives_metrics(tmp_path, capsys):
    from furiosa_opt_engine import _native
    from furiosa_opt_models_b200.bench import forward, metrics

    before = _native._trace_level()
    try:
        _native._trace_flush("/dev/null")
        rc = forward.main(["--model", "tiny-qwen3", "--tier", "gate", "--warmups", "1", "--repetitions", "3",
                           "--out", str(tmp_path), "--profile", "trace"])
    finally:
        _native._trace_set_level(before)
    assert rc == 0
    lines = [json.loads(x) for x in capsys.readouterr().out.splitlines() if x.startswith("{")]
    cases = [x["case"] for x in lines if "case" in x]
    assert cases == ["in-128-out-128-decode-rows-1", "in-128-out-128-decode-rows-16", "in-128-prefill-chunk-128"]
    recs = metrics.collect(str(tmp_path), None)
    step = {r["tags"][2]: r["value"] for r in recs if r["metric"] == "furiosa_opt.forward.step_ms"}
    device = {r["tags"][2]: r["value"] for r in recs if r["metric"] == "furiosa_opt.forward.device_ms"}
    assert set(step) == {f"case:{c}" for c in cases}
    assert set(device) == set(step)
    for c in step:
        assert 0 < device[c] <= step[c] + 0.05
    kernels = [r for r in recs if r["metric"] == "furiosa_opt.kernel.ns"]
    assert {r["tags"][2] for r in kernels} == set(step)
    assert all(r["value"] > 0 for r in kernels)
    assert all(r["tags"][0] == "model:synthetic/tiny-qwen3" and r["tags"][1] == "test:forward" for r in recs)
