"""Catalog compositions: model families that the registry lists but that no kernels serve yet.

Each family is a typed composition built natively from config.json (csrc/engine/catalog.cc): the
module tree and every weight it reads, by checkpoint name and shape, plus the tied copies a
checkpoint may hold or leave out. A checkpoint, or only its safetensors headers
(`Checkpoint.declared`), is checked strictly against it: a missing, misshaped or unread tensor is
refused by name. Loading such a model is still refused by the registry (`NotImplementedError`), as
the reference refuses its catalog families
(crates/furiosa-opt-models/src/models/{encoder,encoder_decoder,decoder/recurrent}).

Families: BERT (`BertModel`), T5 and mT5 (`T5ForConditionalGeneration`,
`MT5ForConditionalGeneration`), Whisper (`WhisperForConditionalGeneration`), Mamba-2
(`Mamba2ForCausalLM`) and Gemma-3 text (`Gemma3ForCausalLM`).
"""

from __future__ import annotations

import dataclasses


@dataclasses.dataclass(frozen=True)
class Composition:
    family: str
    architecture: str
    tree: tuple[str, ...]
    weights: dict[str, tuple[int, ...]]
    aliases: dict[str, tuple[int, ...]]

    def describe(self) -> str:
        return "\n".join(self.tree)

    def parameters(self) -> int:
        total = 0
        for shape in self.weights.values():
            n = 1
            for d in shape:
                n *= d
            total += n
        return total


def composes(architecture: str) -> bool:
    from furiosa_opt_engine import _native

    return bool(_native._catalog_composes(architecture))


def compose(checkpoint, check: bool = True) -> Composition:
    """The composition of `checkpoint`'s config (a `furiosa_opt_engine.Checkpoint`), checked
    against its tensors unless `check` is False. Raises ValueError naming the config key or tensor
    that does not fit."""
    from furiosa_opt_engine import _native

    d = _native._catalog(checkpoint, check)
    return Composition(d["family"], d["architecture"], tuple(d["tree"]), dict(d["weights"]), dict(d["aliases"]))
