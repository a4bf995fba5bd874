"""Benchmarks of the engine's forward calls and the metrics records made from their traces.

- `forward`: the forward-phase cases of the serving workloads (a prompt's last chunk, decode
  steps halfway through the output at each concurrency), timed call by call in a Chrome trace.
- `metrics`: JSONL metric records (step time and kernel time per case, serving latencies) from
  those traces and from `vllm bench serve` summaries.
- `benchmarks.json`: the workloads and the models they run on.
"""

import json as _json
import os as _os

INVENTORY = _os.path.join(_os.path.dirname(__file__), "benchmarks.json")


def inventory() -> dict:
    with open(INVENTORY) as f:
        return _json.load(f)
