"""Options of this plugin inside vLLM's `additional_config`, under the key `furiosa`.

The key and the option names are the reference plugin's public configuration
(integrations/furiosa-opt-vllm/furiosa_opt_vllm/additional.py there); the parser is strict in the
same way: an unknown option or a value of the wrong type is refused, naming its full path.

- `cuda_graphs` (bool, default true): decode calls replay the CUDA graphs the engine captured for
  each call shape; false launches every call eagerly, which profilers prefer.
- `draft_placement` ({"chips": [...], "pes": [start, end]}): where a draft model would run. Here
  the draft model always shares the worker's GPU with the target, so any placement is refused
  once it has been checked for shape.
"""

from __future__ import annotations

import dataclasses

from .admission import Refused

ROOT = "additional_config.furiosa"


def _ordinal(value, path: str) -> int:
    # bool is an int subclass in Python; a flag is not an ordinal.
    if isinstance(value, bool) or not isinstance(value, int):
        raise Refused(path, f"{value!r} is not an integer")
    if value < 0:
        raise Refused(path, f"{value} is negative")
    return value


def _fields(raw, path: str, known: tuple[str, ...]) -> dict:
    if not isinstance(raw, dict):
        raise Refused(path, f"expected a mapping, got {type(raw).__name__}")
    for key in raw:
        if key not in known:
            raise Refused(f"{path}.{key}", f"unknown option (known: {', '.join(known)})")
    return raw


@dataclasses.dataclass(frozen=True)
class Placement:
    """GPU ordinals in rank order, and the half-open range of processing elements `pes` that the
    reference splits one of its chips by (a GPU is never split: one range)."""

    chips: tuple[int, ...]
    pes: tuple[int, int] = (0, 8)

    @classmethod
    def parse(cls, raw, path: str) -> "Placement":
        fields = _fields(raw, path, ("chips", "pes"))
        if "chips" not in fields:
            raise Refused(f"{path}.chips", "required")
        listed = fields["chips"]
        if not isinstance(listed, (list, tuple)) or not listed:
            raise Refused(f"{path}.chips", "a non-empty list of GPU ordinals")
        chips = tuple(_ordinal(c, f"{path}.chips.{i}") for i, c in enumerate(listed))
        repeated = sorted({c for c in chips if chips.count(c) > 1})
        if repeated:
            raise Refused(f"{path}.chips", f"GPU {repeated[0]} appears more than once")
        pes = fields.get("pes", (0, 8))
        if not isinstance(pes, (list, tuple)) or len(pes) != 2:
            raise Refused(f"{path}.pes", "a [start, end) pair")
        return cls(chips, tuple(_ordinal(p, f"{path}.pes.{i}") for i, p in enumerate(pes)))


@dataclasses.dataclass(frozen=True)
class Section:
    """The parsed `furiosa` options; an option that is not given keeps its default."""

    cuda_graphs: bool = True
    draft_placement: Placement | None = None

    @classmethod
    def parse(cls, config) -> "Section":
        """The options in `config.additional_config["furiosa"]` (all defaults without that key). A
        malformed option, or one this engine does not serve, is refused with its path."""
        extra = getattr(config, "additional_config", None) or {}
        raw = extra.get("furiosa", {}) if isinstance(extra, dict) else {}
        fields = _fields(raw, ROOT, ("cuda_graphs", "draft_placement"))
        graphs = fields.get("cuda_graphs", True)
        if not isinstance(graphs, bool):
            raise Refused(f"{ROOT}.cuda_graphs", f"{graphs!r} is not true or false")
        placement = fields.get("draft_placement")
        if placement is not None:
            Placement.parse(placement, f"{ROOT}.draft_placement")
            raise Refused(f"{ROOT}.draft_placement", "a draft model runs beside the target on the worker's GPU")
        return cls(graphs, None)
