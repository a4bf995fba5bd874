"""vLLM pooling requests (embeddings and classification) through the engine's non-token outputs.

- `embed`: a causal checkpoint loads as its base model (`Qwen3ForCausalLM` as `Qwen3Model`), whose
  calls return final-normed hidden rows; a request's prompt is pooled (LAST: its last row, MEAN:
  the mean of its rows, CLS: its first row), truncated to `dimensions` (Matryoshka) and
  L2-normalized unless `use_activation` is False.
- `classify`: a `*ForSequenceClassification` checkpoint returns FP32 label scores of each kept row
  (label columns first); the pooled row's first `num_labels` columns go through softmax (sigmoid
  for one label) unless `use_activation` is False.

These are the pooling heads vLLM applies (vllm/model_executor/layers/pooler/seqwise/heads.py),
done here on the rows the engine returns; the reference plugin runs vLLM's own pooler on the same
rows (integrations/furiosa-opt-vllm/furiosa_opt_vllm/embedding/__init__.py:33-130).
"""

from __future__ import annotations

import torch

from .admission import Refused

TASKS = ("embed", "classify")

# Causal classes served as their base model when vLLM pools their hidden rows.
BASE_MODELS = {"Qwen3ForCausalLM": "Qwen3Model", "Qwen3Model": "Qwen3Model"}


def base_architecture(architecture: str) -> str | None:
    """The architecture a pooling load selects: a classifier as itself, a causal model as its base
    model; None when the checkpoint's class is not served for pooling."""
    if architecture.endswith("ForSequenceClassification"):
        return architecture
    return BASE_MODELS.get(architecture)


def check(task: str | None, served: tuple[str, ...]) -> None:
    if task is not None and task not in served:
        raise Refused("task", f"{task}: this model serves {', '.join(served) or 'no pooling'}")


class Pool:
    """One request's pooling over its prompt chunks."""

    def __init__(self, params, method: str, prompt: int):
        self.params = params
        self.method = (method or "LAST").upper()
        if self.method not in ("LAST", "MEAN", "CLS"):
            raise Refused("pooling_type", f"{method}: LAST, MEAN or CLS pooling is served")
        self.prompt = prompt
        self.sum: torch.Tensor | None = None
        self.first: torch.Tensor | None = None
        self.last: torch.Tensor | None = None

    def keep_all(self, computed: int) -> bool:
        """Whether a chunk starting at `computed` keeps every row (else only the prompt's last)."""
        return self.method == "MEAN" or (self.method == "CLS" and computed == 0)

    def add(self, rows: torch.Tensor, computed: int, n: int) -> None:
        """Rows the engine returned for a chunk of `n` prompt rows after `computed` positions."""
        if self.method == "MEAN":
            s = rows.float().sum(0)
            self.sum = s if self.sum is None else self.sum + s
        elif self.method == "CLS" and computed == 0:
            self.first = rows[0].float()
        if computed + n == self.prompt and rows.shape[0]:
            self.last = rows[-1].float()

    def done(self, computed: int) -> bool:
        return computed >= self.prompt

    def pooled(self) -> torch.Tensor:
        if self.method == "MEAN":
            return self.sum / self.prompt
        if self.method == "CLS":
            return self.first
        return self.last


def embed(pooled: torch.Tensor, params) -> torch.Tensor:
    v = pooled.float()
    d = getattr(params, "dimensions", None)
    if d is not None:
        v = v[:d]
    if getattr(params, "use_activation", None) is not False:
        v = torch.nn.functional.normalize(v, p=2, dim=-1)
    return v


def classify(pooled: torch.Tensor, params, labels: int) -> torch.Tensor:
    v = pooled.float()[:labels]
    if getattr(params, "use_activation", None) is not False:
        v = torch.sigmoid(v) if labels < 2 else torch.softmax(v, dim=-1)
    return v
