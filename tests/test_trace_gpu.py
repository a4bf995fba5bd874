"""Tracing a decoder call on the GPU: at `trace` level every kernel launch becomes a device span
(the call runs eagerly), beside the call's host span and its device span."""

import json

import pytest

pytestmark = pytest.mark.gpu


def test_trace_level_records_kernel_spans(tmp_path):
    import torch

    import furiosa_opt_engine as engine
    from furiosa_opt_engine import _native
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import configs

    before = _native._trace_level()
    _native._trace_set_level("trace")
    try:
        _native._trace_flush("/dev/null")
        cfg = configs.get("tiny-qwen3")
        device = engine.Device(engine.Placement([0], range(8)))
        model = _native._synthetic_decoder(device, cfg, seed=0, std=0.02)
        cache = engine.decoder.Cache(model.cache, 16)
        alloc = serving.BlockAllocator(16)
        prompt = torch.randint(0, cfg["vocab"], (9,), dtype=torch.int32)
        seq = serving.Sequence(engine.HostTensor.from_dlpack(prompt).to_hbm(device), 9, alloc.take(4))
        serving.prefill(model, cache, [seq], [0]).to_host()
        serving.decode(model, cache, [seq]).to_host()
        path = _native._trace_flush(str(tmp_path / "trace.json"))
    finally:
        _native._trace_set_level(before)
    events = json.load(open(path))["traceEvents"]
    calls = [e for e in events if e["name"] == "forward"]
    device_calls = [e for e in events if e["name"] == "forward.device"]
    kernels = [e for e in events if e["cat"] == "GPU" and e["name"] != "forward.device"]
    assert len(calls) == 2 and len(device_calls) == 2
    assert all(e["dur"] > 0 for e in device_calls)
    # Every layer launches its projections: at least 4 GEMM spans a layer a call.
    assert sum(e["name"].startswith("gemm") for e in kernels) >= 2 * 4 * cfg["layers"]
    assert all(e["dur"] >= 0 for e in kernels)
    # The kernels of a call lie within its device span.
    first = device_calls[0]
    inside = [k for k in kernels if first["ts"] - 1 <= k["ts"] <= first["ts"] + first["dur"] + 1]
    assert inside
