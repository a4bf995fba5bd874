"""The plugin's section of vLLM's `additional_config`: the options under its `furiosa` key
(the reference's integrations/furiosa-opt-vllm/furiosa_opt_vllm/additional.py: the same key and
the same strict parsing, with this engine's options).

- `cuda_graphs` (default true): decode calls replay CUDA graphs the engine captured per call
  shape; false runs every call eagerly (for profiling).
- `draft_placement` (the reference's chips for a draft model): a draft model runs beside the
  target on the worker's GPU, so another placement is refused.
"""

from __future__ import annotations

from typing import Annotated, ClassVar

from pydantic import BaseModel, ConfigDict, Field, ValidationError, field_validator

from .admission import Refused

Index = Annotated[int, Field(strict=True, ge=0)]


class Placement(BaseModel):
    """GPU ordinals in rank order, and the half-open range `pes` the reference splits a chip by
    (one range on a GPU)."""

    model_config: ClassVar[ConfigDict] = ConfigDict(frozen=True, extra="forbid")

    chips: tuple[Index, ...]
    pes: tuple[Index, Index] = (0, 8)

    @field_validator("chips")
    @classmethod
    def distinct(cls, chips: tuple[int, ...]) -> tuple[int, ...]:
        seen: set[int] = set()
        for ordinal in chips:
            if ordinal in seen:
                raise ValueError(f"GPU {ordinal} is listed twice")
            seen.add(ordinal)
        if not seen:
            raise ValueError("a placement lists at least one GPU")
        return chips


class Section(BaseModel):
    """Options read from `additional_config["furiosa"]`; an option left out keeps its default."""

    model_config: ClassVar[ConfigDict] = ConfigDict(frozen=True, extra="forbid")

    cuda_graphs: Annotated[bool, Field(strict=True)] = True
    draft_placement: Placement | None = None

    @classmethod
    def parse(cls, config) -> Section:
        """The section of `config`'s `additional_config` (defaults without a `furiosa` key); a
        malformed section or an option the engine does not serve is refused with its path."""
        raw = getattr(config, "additional_config", None) or {}
        try:
            section = cls.model_validate(raw.get("furiosa", {}) if isinstance(raw, dict) else {})
        except ValidationError as e:
            d = e.errors()[0]
            path = ".".join(map(str, ("additional_config", "furiosa", *d["loc"])))
            raise Refused(path, d["msg"]) from None
        if section.draft_placement is not None:
            raise Refused("additional_config.furiosa.draft_placement",
                          "a draft model runs beside the target on the worker's GPU")
        return section
