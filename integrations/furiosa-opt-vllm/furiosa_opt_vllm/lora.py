"""vLLM's LoRA adapters as engine adapters (the reference's behaviour:
integrations/furiosa-opt-vllm/furiosa_opt_vllm/lora.py).

- Loaded adapters, by LoRA ID: the worker's `add_lora`, or a step whose request names an adapter,
  reads the adapter's PEFT checkpoint onto the device (again when the request loads in place).
  Up to `max_cpu_loras` (else `max_loras`) stay loaded, least recently used out first.
- Slots: the adapters list every engine call takes, `max_loras` of them (at most the engine's
  SLOTS). Each engine request names its sequence's slot.
- A pinned adapter stays loaded and in its slot until removed. Making room never evicts a pinned
  adapter or one the step runs; when only such adapters could make room the call is refused before
  anything changes.
"""

from __future__ import annotations

import json
from collections import OrderedDict
from pathlib import Path


class Adapters:
    def __init__(self, max_loras: int, max_cpu_loras: int | None, spec, read=None):
        self.max_loras = max_loras
        self.capacity = max_cpu_loras or max_loras
        self.spec = spec
        self._read_fn = read  # (lora_request) -> engine adapter; tests give their own
        self.loaded: OrderedDict[int, object] = OrderedDict()  # LoRA ID -> adapter, LRU first
        self.held: OrderedDict[int, int] = OrderedDict()  # LoRA ID -> slot, LRU first
        self.pins: set[int] = set()
        self.slots: list = [None] * max_loras

    # ---------------------------------------------------------------- worker API
    def add(self, request, keep: frozenset = frozenset()) -> bool:
        lid = request.lora_int_id
        unload, displace = self._room(lid, keep)
        if lid not in self.loaded or getattr(request, "load_inplace", False):
            adapter = self._read(request)
            if unload is not None:
                self.remove(unload)
            self.loaded[lid] = adapter
        self.loaded.move_to_end(lid)
        self._hold(lid, displace)
        return True

    def remove(self, lid: int) -> bool:
        self.pins.discard(lid)
        slot = self.held.pop(lid, None)
        if slot is not None:
            self.slots[slot] = None
        return self.loaded.pop(lid, None) is not None

    def pin(self, lid: int) -> bool:
        if lid not in self.loaded:
            raise ValueError(f"LoRA adapter {lid} is not loaded")
        _, displace = self._room(lid, frozenset())
        self._hold(lid, displace)
        self.pins.add(lid)
        return True

    def ids(self) -> set[int]:
        return set(self.loaded)

    # ---------------------------------------------------------------- a step
    def activate(self, named: dict) -> dict:
        """The slot of each request ID in `named` (request ID -> LoRA request), once every adapter
        of the step is loaded and holds a slot."""
        adapters = {r.lora_int_id: r for r in named.values()}
        if len(adapters) > self.max_loras:
            raise RuntimeError(f"a step runs {len(adapters)} adapters, above --max-loras")
        step = frozenset(adapters)
        for r in adapters.values():
            self.add(r, step)
        return {rid: self.held[r.lora_int_id] for rid, r in named.items()}

    # ---------------------------------------------------------------- room
    def _room(self, lid: int, keep: frozenset):
        kept = self.pins | set(keep) | {lid}
        unload = None
        if lid not in self.loaded and len(self.loaded) >= self.capacity:
            unload = next((o for o in self.loaded if o not in kept), None)
            if unload is None:
                raise RuntimeError(f"LoRA adapter {lid}: the {self.capacity} loaded adapters are pinned or in use; "
                                   "raise --max-cpu-loras")
        holders = [o for o in self.held if o != unload]
        displace = None
        if lid not in self.held and len(holders) >= self.max_loras:
            displace = next((o for o in holders if o not in kept), None)
            if displace is None:
                raise RuntimeError(f"LoRA adapter {lid}: pinned or running adapters hold every slot; raise --max-loras")
        return unload, displace

    def _hold(self, lid: int, displace) -> None:
        if displace is not None:
            self.slots[self.held.pop(displace)] = None
        slot = self.held.pop(lid, None)
        if slot is None:
            slot = min(set(range(self.max_loras)) - set(self.held.values()))
        self.held[lid] = slot
        self.slots[slot] = self.loaded[lid]

    def _read(self, request):
        if self._read_fn is not None:
            return self._read_fn(request)
        import furiosa_opt_engine as engine

        if getattr(request, "tensorizer_config_dict", None) is not None:
            raise ValueError(f"LoRA adapter {request.lora_name}: reads no tensorizer checkpoint")
        path = Path(request.lora_path)
        if not (path / "adapter_model.safetensors").is_file():
            raise ValueError(f"LoRA adapter {request.lora_name}: reads adapter_model.safetensors")
        config = json.loads((path / "adapter_config.json").read_text())
        return engine.decoder.Adapter(self.spec, engine.Checkpoint(str(path), config))
