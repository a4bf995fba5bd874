"""FP32 PyTorch forwards of catalog families on the host, reading a checkpoint by the names its
catalog composition checked (csrc/engine/catalog.cc): the oracles that kernels for these families
will be tested against, and a CPU path for small encoders.

- `encoder`: BERT and XLM-RoBERTa (BGE-M3) encoders, post-norm layers with exact GELU: the final
  hidden rows of each sequence and, where the composition has one, the pooled first row.
"""

from __future__ import annotations

import json
import math
import os

import torch


def load_tensors(directory: str) -> dict[str, torch.Tensor]:
    """Every tensor of the directory's safetensors files, as FP32."""
    from safetensors.torch import load_file

    out: dict[str, torch.Tensor] = {}
    for name in sorted(os.listdir(directory)):
        if name.endswith(".safetensors"):
            out.update({k: v.float() for k, v in load_file(os.path.join(directory, name)).items()})
    return out


def _layer_norm(x, w, b, eps):
    return torch.nn.functional.layer_norm(x, (x.shape[-1],), w, b, eps)


def encoder(directory: str, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None,
            token_type_ids: torch.Tensor | None = None):
    """(hidden [batch, tokens, hidden], pooled [batch, hidden] or None) of a BERT or XLM-RoBERTa
    checkpoint; `attention_mask` (1 for real tokens) keeps padding out of every row's attention."""
    import furiosa_opt_engine as engine

    from . import catalog

    comp = catalog.compose(engine.Checkpoint(directory))
    if comp.family not in ("bert", "xlm_roberta"):
        raise ValueError(f"{comp.architecture}: not a BERT-style encoder")
    with open(os.path.join(directory, "config.json")) as f:
        cfg = json.load(f)
    t = load_tensors(directory)
    p = next(k for k in comp.weights if k.endswith("embeddings.word_embeddings.weight"))[: -len("embeddings.word_embeddings.weight")]
    eps = float(cfg.get("layer_norm_eps", 1e-12))
    heads = int(cfg["num_attention_heads"])
    ids = input_ids.long()
    batch, n = ids.shape
    mask = torch.ones_like(ids) if attention_mask is None else attention_mask.long()
    types = torch.zeros_like(ids) if token_type_ids is None else token_type_ids.long()
    if comp.family == "xlm_roberta":
        # RoBERTa numbers real tokens from padding_idx + 1; padding keeps padding_idx.
        pad = int(cfg.get("pad_token_id", 1))
        positions = torch.cumsum(mask, dim=1) * mask + pad
    else:
        positions = torch.arange(n).expand(batch, n)
    x = (t[p + "embeddings.word_embeddings.weight"][ids] + t[p + "embeddings.position_embeddings.weight"][positions]
         + t[p + "embeddings.token_type_embeddings.weight"][types])
    x = _layer_norm(x, t[p + "embeddings.LayerNorm.weight"], t[p + "embeddings.LayerNorm.bias"], eps)
    bias = (1.0 - mask[:, None, None, :].float()) * torch.finfo(torch.float32).min
    layers = int(cfg["num_hidden_layers"])
    for layer in range(layers):
        q = p + f"encoder.layer.{layer}."

        def lin(name, v):
            return v @ t[q + name + ".weight"].T + t[q + name + ".bias"]

        d = x.shape[-1] // heads
        split = lambda v: v.view(batch, n, heads, d).transpose(1, 2)  # noqa: E731
        qs, ks, vs = (split(lin(f"attention.self.{m}", x)) for m in ("query", "key", "value"))
        att = torch.softmax(qs @ ks.transpose(-1, -2) / math.sqrt(d) + bias, dim=-1) @ vs
        att = att.transpose(1, 2).reshape(batch, n, heads * d)
        x = _layer_norm(x + lin("attention.output.dense", att), t[q + "attention.output.LayerNorm.weight"],
                        t[q + "attention.output.LayerNorm.bias"], eps)
        mid = torch.nn.functional.gelu(lin("intermediate.dense", x))
        x = _layer_norm(x + lin("output.dense", mid), t[q + "output.LayerNorm.weight"], t[q + "output.LayerNorm.bias"],
                        eps)
    pooled = None
    if p + "pooler.dense.weight" in t and (p + "pooler.dense.weight" in comp.weights or
                                             p + "pooler.dense.weight" in comp.optional):
        pooled = torch.tanh(x[:, 0] @ t[p + "pooler.dense.weight"].T + t[p + "pooler.dense.bias"])
    return x, pooled
