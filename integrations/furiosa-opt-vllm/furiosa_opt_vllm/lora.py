"""vLLM LoRA requests served as engine adapters.

The engine takes a fixed list of adapter slots with every call (``decoder.adapters`` of them) and
each engine request names the slot of its adapter. vLLM names adapters by LoRA ID and may ask for
more of them than fit on the device. This module keeps:

- a table of loaded adapters (LoRA ID -> engine adapter, the clock tick of its last use and its
  pin), at most ``max_cpu_loras`` (else ``max_loras``) entries;
- a lease per engine slot (the LoRA ID that holds it), ``max_loras`` slots.

Whenever an adapter has to come in, the entry (or lease) with the oldest tick that is neither
pinned nor needed by the current step goes out. Every decision is made before anything changes,
so a refused step leaves the table as it was. Behaviour follows the reference plugin's LoRA
support (integrations/furiosa-opt-vllm/furiosa_opt_vllm/lora.py there): LRU unloading, pins that
keep their slot, and refusal when only pinned or running adapters could make room.
"""

from __future__ import annotations

import dataclasses
import itertools
import json
from pathlib import Path


@dataclasses.dataclass
class _Entry:
    adapter: object
    tick: int
    pinned: bool = False


class Adapters:
    """LoRA adapters of one worker: loaded entries and the engine's slot leases."""

    def __init__(self, max_loras: int, max_cpu_loras: int | None, spec, read=None):
        self.max_loras = max_loras
        self.capacity = max_cpu_loras or max_loras
        self.spec = spec
        self._reader = read  # lora_request -> engine adapter (tests pass their own)
        self._entries: dict[int, _Entry] = {}
        self._lease: list[int | None] = [None] * max_loras  # LoRA ID holding each slot
        self._clock = itertools.count(1)

    # ------------------------------------------------------------------ what the engine call takes
    @property
    def slots(self) -> list:
        """The engine adapter in each slot (None for a free slot), in slot order."""
        return [None if lid is None else self._entries[lid].adapter for lid in self._lease]

    def slot_of(self, lid: int) -> int | None:
        return self._lease.index(lid) if lid in self._lease else None

    # ------------------------------------------------------------------ the worker's LoRA calls
    def add(self, request, step: frozenset = frozenset()) -> bool:
        """Loads `request`'s adapter (again when it asks to load in place) and gives it a slot."""
        lid = request.lora_int_id
        protected = step | {lid}
        unload = None
        if lid not in self._entries and len(self._entries) >= self.capacity:
            unload = self._oldest(self._entries, protected)
            if unload is None:
                raise RuntimeError(f"LoRA adapter {lid} cannot load: the {self.capacity} loaded adapters are "
                                   "pinned or used by this step (raise --max-cpu-loras)")
        slot = self._plan_slot(lid, protected, freed=unload)
        if lid not in self._entries or getattr(request, "load_inplace", False):
            adapter = self._read(request)  # may raise: nothing has changed yet
            if unload is not None:
                self.remove(unload)
            if lid in self._entries:
                self._entries[lid].adapter = adapter
            else:
                self._entries[lid] = _Entry(adapter, 0)
        self._take(lid, slot)
        return True

    def remove(self, lid: int) -> bool:
        slot = self.slot_of(lid)
        if slot is not None:
            self._lease[slot] = None
        return self._entries.pop(lid, None) is not None

    def pin(self, lid: int) -> bool:
        if lid not in self._entries:
            raise ValueError(f"LoRA adapter {lid} is not loaded")
        self._take(lid, self._plan_slot(lid, frozenset({lid})))
        self._entries[lid].pinned = True
        return True

    def ids(self) -> set[int]:
        return set(self._entries)

    # ------------------------------------------------------------------ a step
    def activate(self, named: dict) -> dict:
        """Loads and seats every adapter a step names (request ID -> LoRA request); returns each
        request ID's slot."""
        wanted = {r.lora_int_id: r for r in named.values()}
        if len(wanted) > self.max_loras:
            raise RuntimeError(f"a step runs {len(wanted)} adapters, above --max-loras ({self.max_loras})")
        step = frozenset(wanted)
        for r in wanted.values():
            self.add(r, step)
        return {rid: self.slot_of(r.lora_int_id) for rid, r in named.items()}

    # ------------------------------------------------------------------ bookkeeping
    def _oldest(self, ids, protected) -> int | None:
        """The least recently used of `ids` that is neither pinned nor protected."""
        free = [i for i in ids if i not in protected and not self._entries[i].pinned]
        return min(free, key=lambda i: self._entries[i].tick) if free else None

    def _plan_slot(self, lid: int, protected, freed: int | None = None) -> int:
        """The slot `lid` will hold: its own, else the lowest free one (or the one `freed` gives
        up), else the lease of the least recently used unprotected holder."""
        own = self.slot_of(lid)
        if own is not None:
            return own
        for s, holder in enumerate(self._lease):
            if holder is None or holder == freed:
                return s
        victim = self._oldest([h for h in self._lease if h is not None], protected)
        if victim is None:
            raise RuntimeError(f"LoRA adapter {lid} gets no slot: pinned or running adapters hold every "
                               "slot (raise --max-loras)")
        return self._lease.index(victim)

    def _take(self, lid: int, slot: int) -> None:
        own = self.slot_of(lid)
        if own is not None and own != slot:
            self._lease[own] = None
        self._lease[slot] = lid
        self._entries[lid].tick = next(self._clock)

    def _read(self, request):
        if self._reader is not None:
            return self._reader(request)
        import furiosa_opt_engine as engine

        if getattr(request, "tensorizer_config_dict", None) is not None:
            raise ValueError(f"LoRA adapter {request.lora_name}: tensorizer checkpoints are not read, only PEFT")
        path = Path(request.lora_path)
        if not (path / "adapter_model.safetensors").is_file():
            raise ValueError(f"LoRA adapter {request.lora_name}: no adapter_model.safetensors in {path}")
        config = json.loads((path / "adapter_config.json").read_text())
        return engine.decoder.Adapter(self.spec, engine.Checkpoint(str(path), config))
