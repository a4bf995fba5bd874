"""Tracing: FURIOSA_OPT_PROFILE levels and the Chrome trace the engine writes (host spans here; the
device spans of a decoder call in tests/test_trace_gpu.py)."""

import json

import pytest

from furiosa_opt_engine import _native


@pytest.fixture
def level():
    before = _native._trace_level()
    yield
    _native._trace_set_level(before)
    _native._trace_flush("/dev/null")


def test_host_spans_become_a_chrome_trace(tmp_path, level):
    _native._trace_set_level("info")
    assert _native._trace_level() == "info"
    t0 = _native._trace_now_ns()
    _native._trace_span("schedule", "framework", t0, t0 + 1500)
    _native._trace_span("sample", "framework", t0 + 2000, t0 + 2500)
    path = _native._trace_flush(str(tmp_path / "t.json"))
    assert path == str(tmp_path / "t.json")
    events = json.load(open(path))["traceEvents"]
    assert [e["name"] for e in events] == ["schedule", "sample"]
    assert all(e["ph"] == "X" and e["cat"] == "framework" for e in events)
    assert events[0]["dur"] == pytest.approx(1.5)
    assert events[1]["ts"] - events[0]["ts"] == pytest.approx(2.0)
    # Flushing cleared them: nothing left to write.
    assert _native._trace_flush(str(tmp_path / "u.json")) == ""


def test_levels(level):
    for name in ("off", "info", "debug", "trace"):
        _native._trace_set_level(name)
        assert _native._trace_level() == name
    with pytest.raises(ValueError, match="a trace level is off, info, debug or trace"):
        _native._trace_set_level("verbose")
