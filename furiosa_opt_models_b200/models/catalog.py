"""Catalog compositions: model families that the registry lists but that no kernels serve yet.

Each family is a typed composition built natively from config.json (csrc/engine/catalog.cc): the
module tree and every weight it reads, by checkpoint name and shape, plus the weights a checkpoint
may hold or leave out (tied copies, unused parts) and the names nothing reads (old buffers,
pretraining heads). A checkpoint, or only its safetensors headers
(`Checkpoint.declared`), is checked strictly against it: a missing, misshaped or unread tensor is
refused by name. Loading such a model is still refused by the registry (`NotImplementedError`), as
the reference refuses its catalog families
(crates/furiosa-opt-models/src/models/{encoder,encoder_decoder,vision_language,decoder/recurrent,
decoder/hybrid,decoder/attention}).

Families (`architectures()` lists every name): BERT and its classification and masked-LM heads,
XLM-RoBERTa (BGE-M3, rerankers), CLIP and SigLIP, T5 / mT5, Whisper, Mamba, Mamba-2, Bamba,
Gemma-3 and Gemma-4 text, OLMoE, DeepSeek-V2, LLaVA, Mllama and Qwen3-VL.
"""

from __future__ import annotations

import dataclasses


@dataclasses.dataclass(frozen=True)
class Composition:
    family: str
    architecture: str
    tree: tuple[str, ...]
    weights: dict[str, tuple[int, ...]]
    optional: dict[str, tuple[int, ...]]
    ignored: tuple[str, ...]

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


def architectures() -> list[str]:
    from furiosa_opt_engine import _native

    return list(_native._catalog_architectures())


def compose(checkpoint, check: bool = True) -> Composition:
    """The composition of `checkpoint`'s config (a `furiosa_opt_engine.Checkpoint`), checked
    against its tensors unless `check` is False. Raises ValueError naming the config key or tensor
    that does not fit."""
    from furiosa_opt_engine import _native

    d = _native._catalog(checkpoint, check)
    return Composition(d["family"], d["architecture"], tuple(d["tree"]), dict(d["weights"]), dict(d["optional"]),
                       tuple(d["ignored"]))
