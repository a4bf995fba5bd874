"""Loading of the native extension and the per-device scratch its kernels share."""

from __future__ import annotations

import importlib
import threading

import torch

_lock = threading.Lock()
_native = None


def native():
    """The ``furiosa_opt_engine._native`` module; raises ImportError when it is not built."""
    global _native
    if _native is None:
        with _lock:
            if _native is None:
                _native = importlib.import_module("furiosa_opt_engine._native")
    return _native


class Scratch:
    """Device scratch of one GPU: split-K partials, arrival counters (kept zero between launches)
    and the status word kernels write instead of hanging."""

    def __init__(self, device: torch.device, workspace_bytes: int = 64 << 20, counters: int = 65536):
        self.device = device
        self.workspace = torch.empty(workspace_bytes // 4, dtype=torch.float32, device=device)
        self.counters = torch.zeros(counters, dtype=torch.int32, device=device)
        self.status = torch.zeros(4, dtype=torch.int32, device=device)

    def check(self) -> None:
        """Raises RuntimeError when a kernel recorded a failure since the last check."""
        code = int(self.status[0].item())
        if code != 0:
            self.status.zero_()
            raise RuntimeError(f"kernel reported status {code} (a bounded wait gave up)")


_scratch: dict[int, Scratch] = {}


def scratch(device: torch.device | None = None) -> Scratch:
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    index = device.index if device.index is not None else torch.cuda.current_device()
    s = _scratch.get(index)
    if s is None:
        s = _scratch[index] = Scratch(torch.device("cuda", index))
    return s
