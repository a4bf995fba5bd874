"""Engine log records reach Python's `logging` (logger "furiosa_opt_engine") when a binding call
returns: checkpoint opens at DEBUG, trace writes at INFO, and a full queue keeps the newest records
and says how many it dropped."""

import json
import logging

from furiosa_opt_engine import _native

import furiosa_opt_engine as engine


def test_records_reach_python_logging(caplog):
    with caplog.at_level(logging.DEBUG, logger="furiosa_opt_engine"):
        _native._log(logging.WARNING, "a warning from the engine")
    assert [(r.name, r.levelno, r.getMessage()) for r in caplog.records] == [
        ("furiosa_opt_engine", logging.WARNING, "a warning from the engine")]


def test_checkpoint_open_logs_its_tensor_count(tmp_path, caplog):
    import torch
    from safetensors.torch import save_file

    (tmp_path / "config.json").write_text(json.dumps({"architectures": ["X"]}))
    save_file({"a.weight": torch.zeros(2, 2), "b.weight": torch.zeros(3)}, str(tmp_path / "model.safetensors"))
    with caplog.at_level(logging.DEBUG, logger="furiosa_opt_engine"):
        engine.Checkpoint(str(tmp_path))
    assert any(r.levelno == logging.DEBUG and r.getMessage().endswith(": 2 tensors") for r in caplog.records)


def test_trace_flush_logs_the_path(tmp_path, caplog):
    t0 = _native._trace_now_ns()
    _native._trace_span("phase", "host", t0, t0 + 1000, "{}")
    with caplog.at_level(logging.INFO, logger="furiosa_opt_engine"):
        path = _native._trace_flush(str(tmp_path / "t.json"))
    assert path and any(r.getMessage() == f"trace written to {path}" for r in caplog.records)


def test_a_full_queue_keeps_the_newest_records(caplog):
    with caplog.at_level(logging.INFO, logger="furiosa_opt_engine"):
        _native._log(logging.INFO, "record", 1030)
    messages = [r.getMessage() for r in caplog.records]
    assert messages[0] == "6 older engine log records were dropped (queue full)"
    assert messages[1:] == ["record"] * 1024


def test_records_below_the_logger_level_are_not_shown(caplog):
    with caplog.at_level(logging.WARNING, logger="furiosa_opt_engine"):
        _native._log(logging.INFO, "quiet")
    assert not caplog.records
