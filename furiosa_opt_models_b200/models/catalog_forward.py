"""FP32 PyTorch forwards of catalog families on the host, reading a checkpoint by the names its
catalog composition checked (csrc/engine/catalog.cc): the oracles that kernels for these families
will be tested against, and a CPU path for small encoders.

- `encoder`: BERT and XLM-RoBERTa (BGE-M3) encoders, post-norm layers with exact GELU: the final
  hidden rows of each sequence and, where the composition has one, the pooled first row.
- `t5_encoder`: the T5 / mT5 encoder stack (RMSNorm before each block, unscaled attention with
  bidirectional relative-position buckets from the first block, ReLU or gated-GELU feed-forward):
  final hidden rows, as a diffusion pipeline's text encoder reads them.
- `whisper_encoder`: Whisper's audio encoder (two convolutions over log-mel frames, learned
  positions, pre-norm layers, final LayerNorm): the rows its decoder cross-attends.
- `clip`: CLIP's text and image embeddings (pre-norm towers with quick-GELU, the text tower's
  causal mask and end-of-text row, the image tower's class row, the projections), L2-normalised.
- `gemma3`: a Gemma-3 text decoder's logits (scaled embedding, RMSNorms with a (1 + weight) scale
  around attention and MLP, QK RMSNorm, global layers and sliding-window layers with their own
  RoPE bases, GeGLU MLP).
- `gemma4`: a Gemma-4 text decoder's logits (per-layer input embeddings gated into every layer,
  wider global heads with proportional RoPE, unscaled QK-normed attention, value RMSNorm, keys as
  values where configured, a learned scalar a layer); the mixture-of-experts block is not covered.
- `olmoe`: an OLMoE mixture-of-experts decoder's logits (RMSNorm over the whole q and k
  projections, softmax router, top-k experts combined by their probabilities).
- `deepseek_v2`: a DeepSeek-V2 decoder's logits (multi-head latent attention: low-rank KV with a
  shared rotary key, optional low-rank queries, interleaved RoPE on the rotary dims; routed experts
  by greedy or group-limited top-k, scaled, plus shared experts after the first dense layers).
- `mamba`: a Mamba (1) language model's logits, its selective scan run as the per-channel
  recurrence (state[c] <- exp(dt[c] A[c]) state[c] + dt[c] x[c] B, y[c] = state[c] C + D[c] x[c]).
- `bamba`: a Bamba hybrid's logits: Mamba-2 mixers, and attention with partial RoPE at the
  config's layers, each followed by a gated MLP.
- `mamba2`: a Mamba-2 language model's logits, its selective scan run token by token as the
  recurrence it is (state[h] <- exp(dt A[h]) state[h] + dt x[h] B^T, y[h] = state[h] C + D[h] x[h]),
  the oracle of a future chunked (SSD) scan kernel.
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


def _rms(x, w, eps):
    return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


def mamba2(directory: str, input_ids: torch.Tensor) -> torch.Tensor:
    """Logits [tokens, vocab] of a Mamba-2 checkpoint for one sequence of `input_ids`."""
    import furiosa_opt_engine as engine

    from . import catalog

    comp = catalog.compose(engine.Checkpoint(directory))
    if comp.family != "mamba2":
        raise ValueError(f"{comp.architecture}: not a Mamba-2 model")
    with open(os.path.join(directory, "config.json")) as f:
        cfg = json.load(f)
    t = load_tensors(directory)
    d = int(cfg["hidden_size"])
    inner = int(cfg.get("expand", 2)) * d
    heads, groups, state = int(cfg["num_heads"]), int(cfg.get("n_groups", 1)), int(cfg["state_size"])
    eps = float(cfg.get("layer_norm_epsilon", 1e-5))
    lo, hi = _step_limit(cfg)
    x = t["backbone.embeddings.weight"][input_ids.long().view(-1)]
    for layer in range(int(cfg["num_hidden_layers"])):
        p = f"backbone.layers.{layer}."
        m = p + "mixer."
        x = x + _mamba2_mixer(t, m, _rms(x, t[p + "norm.weight"], eps), inner, heads, groups, state, eps, lo, hi)
    x = _rms(x, t["backbone.norm_f.weight"], eps)
    head = t.get("lm_head.weight", t["backbone.embeddings.weight"])
    return x @ head.T


def _clip_tower(t, p, cfg, x, causal: bool):
    """Pre-norm CLIP layers over rows x [batch, n, d]."""
    heads = int(cfg.get("num_attention_heads", 8))
    eps = float(cfg.get("layer_norm_eps", 1e-5))
    act = cfg.get("hidden_act", "quick_gelu")
    batch, n, d = x.shape
    hd = d // heads
    bias = torch.triu(torch.full((n, n), float("-inf")), 1) if causal else None
    for layer in range(int(cfg["num_hidden_layers"])):
        q = f"{p}encoder.layers.{layer}."

        def lin(name, v):
            return v @ t[q + name + ".weight"].T + t[q + name + ".bias"]

        h = _layer_norm(x, t[q + "layer_norm1.weight"], t[q + "layer_norm1.bias"], eps)
        split = lambda v: v.view(batch, n, heads, hd).transpose(1, 2)  # noqa: E731
        qs, ks, vs = (split(lin(f"self_attn.{m}_proj", h)) for m in ("q", "k", "v"))
        scores = qs @ ks.transpose(-1, -2) / math.sqrt(hd)
        if bias is not None:
            scores = scores + bias
        att = (torch.softmax(scores, dim=-1) @ vs).transpose(1, 2).reshape(batch, n, d)
        x = x + lin("self_attn.out_proj", att)
        h = _layer_norm(x, t[q + "layer_norm2.weight"], t[q + "layer_norm2.bias"], eps)
        h = lin("mlp.fc1", h)
        h = h * torch.sigmoid(1.702 * h) if act == "quick_gelu" else torch.nn.functional.gelu(h)
        x = x + lin("mlp.fc2", h)
    return x


def clip(directory: str, input_ids: torch.Tensor | None = None, pixels: torch.Tensor | None = None):
    """(text embeddings [batch, proj] or None, image embeddings [batch, proj] or None) of a
    `CLIPModel` checkpoint, L2-normalised; `pixels` are [batch, channels, size, size]."""
    import furiosa_opt_engine as engine

    from . import catalog

    comp = catalog.compose(engine.Checkpoint(directory))
    if comp.architecture != "CLIPModel":
        raise ValueError(f"{comp.architecture}: not a CLIPModel")
    with open(os.path.join(directory, "config.json")) as f:
        cfg = json.load(f)
    t = load_tensors(directory)
    text = image = None
    if input_ids is not None:
        tc = cfg.get("text_config", {})
        ids = input_ids.long()
        n = ids.shape[1]
        x = t["text_model.embeddings.token_embedding.weight"][ids] + t["text_model.embeddings.position_embedding.weight"][:n]
        x = _clip_tower(t, "text_model.", tc, x, causal=True)
        x = _layer_norm(x, t["text_model.final_layer_norm.weight"], t["text_model.final_layer_norm.bias"],
                        float(tc.get("layer_norm_eps", 1e-5)))
        eos = int(tc.get("eos_token_id", 2))
        # The end-of-text row: the first eos token (the highest id for configs that predate it).
        rows = (ids == eos).int().argmax(-1) if eos != 2 else ids.argmax(-1)
        text = x[torch.arange(ids.shape[0]), rows] @ t["text_projection.weight"].T
        text = torch.nn.functional.normalize(text, dim=-1)
    if pixels is not None:
        vc = cfg.get("vision_config", {})
        w = t["vision_model.embeddings.patch_embedding.weight"]
        patch = w.shape[-1]
        x = torch.nn.functional.conv2d(pixels.float(), w, stride=patch).flatten(2).transpose(1, 2)
        cls = t["vision_model.embeddings.class_embedding"].expand(x.shape[0], 1, -1)
        x = torch.cat([cls, x], dim=1) + t["vision_model.embeddings.position_embedding.weight"]
        eps = float(vc.get("layer_norm_eps", 1e-5))
        x = _layer_norm(x, t["vision_model.pre_layrnorm.weight"], t["vision_model.pre_layrnorm.bias"], eps)
        x = _clip_tower(t, "vision_model.", vc, x, causal=False)
        pooled = _layer_norm(x[:, 0], t["vision_model.post_layernorm.weight"], t["vision_model.post_layernorm.bias"], eps)
        image = torch.nn.functional.normalize(pooled @ t["visual_projection.weight"].T, dim=-1)
    return text, image


def _t5_buckets(n: int, buckets: int, max_distance: int) -> torch.Tensor:
    """Bidirectional relative-position buckets [n, n] (Raffel et al. 2020): half the buckets a
    direction, exact for small distances, logarithmic up to `max_distance`."""
    rel = torch.arange(n)[None, :] - torch.arange(n)[:, None]  # key - query
    half = buckets // 2
    out = (rel > 0).long() * half
    dist = rel.abs()
    exact = half // 2
    log = exact + (torch.log(dist.float().clamp(min=1) / exact) / math.log(max_distance / exact)
                   * (half - exact)).long()
    log = torch.minimum(log, torch.full_like(log, half - 1))
    return out + torch.where(dist < exact, dist, log)


def t5_encoder(directory: str, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Final hidden rows [batch, tokens, d_model] of a T5 / mT5 checkpoint's encoder."""
    import furiosa_opt_engine as engine

    from . import catalog

    comp = catalog.compose(engine.Checkpoint(directory))
    if comp.family != "t5":
        raise ValueError(f"{comp.architecture}: not a T5 model")
    with open(os.path.join(directory, "config.json")) as f:
        cfg = json.load(f)
    t = load_tensors(directory)
    heads, dkv = int(cfg["num_heads"]), int(cfg["d_kv"])
    eps = float(cfg.get("layer_norm_epsilon", 1e-6))
    gated = str(cfg.get("feed_forward_proj", "relu")).startswith("gated-")
    ids = input_ids.long()
    batch, n = ids.shape
    mask = torch.ones_like(ids) if attention_mask is None else attention_mask.long()

    def norm(x, w):
        return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))

    x = t["shared.weight"][ids]
    rel = t["encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight"]  # [buckets, heads]
    buckets = _t5_buckets(n, rel.shape[0], int(cfg.get("relative_attention_max_distance", 128)))
    bias = rel[buckets].permute(2, 0, 1)[None] + (1.0 - mask[:, None, None, :].float()) * torch.finfo(torch.float32).min
    for layer in range(int(cfg["num_layers"])):
        p = f"encoder.block.{layer}.layer."
        h = norm(x, t[p + "0.layer_norm.weight"])
        split = lambda v: v.view(batch, n, heads, dkv).transpose(1, 2)  # noqa: E731
        q, k, v = (split(h @ t[f"{p}0.SelfAttention.{m}.weight"].T) for m in ("q", "k", "v"))
        att = torch.softmax(q @ k.transpose(-1, -2) + bias, dim=-1) @ v
        x = x + att.transpose(1, 2).reshape(batch, n, heads * dkv) @ t[p + "0.SelfAttention.o.weight"].T
        h = norm(x, t[p + "1.layer_norm.weight"])
        ff = p + "1.DenseReluDense."
        if gated:
            mid = torch.nn.functional.gelu(h @ t[ff + "wi_0.weight"].T, approximate="tanh") * (h @ t[ff + "wi_1.weight"].T)
        else:
            mid = torch.relu(h @ t[ff + "wi.weight"].T)
        x = x + mid @ t[ff + "wo.weight"].T
    return norm(x, t["encoder.final_layer_norm.weight"])


def whisper_encoder(directory: str, features: torch.Tensor) -> torch.Tensor:
    """Encoder rows [batch, frames / 2, d_model] of a Whisper checkpoint for log-mel `features`
    [batch, mel bins, frames]."""
    import furiosa_opt_engine as engine

    from . import catalog

    comp = catalog.compose(engine.Checkpoint(directory))
    if comp.family != "whisper":
        raise ValueError(f"{comp.architecture}: not a Whisper model")
    with open(os.path.join(directory, "config.json")) as f:
        cfg = json.load(f)
    t = load_tensors(directory)
    p = "model.encoder."
    x = torch.nn.functional.gelu(torch.nn.functional.conv1d(features.float(), t[p + "conv1.weight"],
                                                            t[p + "conv1.bias"], padding=1))
    x = torch.nn.functional.gelu(torch.nn.functional.conv1d(x, t[p + "conv2.weight"], t[p + "conv2.bias"], stride=2,
                                                            padding=1))
    x = x.transpose(1, 2)
    batch, n, d = x.shape
    x = x + t[p + "embed_positions.weight"][:n]
    heads = int(cfg["encoder_attention_heads"])
    hd = d // heads
    for layer in range(int(cfg["encoder_layers"])):
        q = f"{p}layers.{layer}."
        h = _layer_norm(x, t[q + "self_attn_layer_norm.weight"], t[q + "self_attn_layer_norm.bias"], 1e-5)
        split = lambda v: v.view(batch, n, heads, hd).transpose(1, 2)  # noqa: E731
        qs = split(h @ t[q + "self_attn.q_proj.weight"].T + t[q + "self_attn.q_proj.bias"])
        ks = split(h @ t[q + "self_attn.k_proj.weight"].T)  # keys carry no bias
        vs = split(h @ t[q + "self_attn.v_proj.weight"].T + t[q + "self_attn.v_proj.bias"])
        att = torch.softmax(qs @ ks.transpose(-1, -2) / math.sqrt(hd), dim=-1) @ vs
        att = att.transpose(1, 2).reshape(batch, n, d)
        x = x + att @ t[q + "self_attn.out_proj.weight"].T + t[q + "self_attn.out_proj.bias"]
        h = _layer_norm(x, t[q + "final_layer_norm.weight"], t[q + "final_layer_norm.bias"], 1e-5)
        h = torch.nn.functional.gelu(h @ t[q + "fc1.weight"].T + t[q + "fc1.bias"])
        x = x + h @ t[q + "fc2.weight"].T + t[q + "fc2.bias"]
    return _layer_norm(x, t[p + "layer_norm.weight"], t[p + "layer_norm.bias"], 1e-5)


def _causal_conv(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None) -> torch.Tensor:
    """Depthwise causal convolution of rows x [n, channels] with kernels w [channels, k], then SiLU."""
    k = w.shape[1]
    padded = torch.cat([torch.zeros(k - 1, x.shape[1]), x])
    out = torch.stack([(padded[i : i + k] * w.T).sum(0) for i in range(x.shape[0])])
    return torch.nn.functional.silu(out if b is None else out + b)


def mamba(directory: str, input_ids: torch.Tensor) -> torch.Tensor:
    """Logits [tokens, vocab] of a Mamba checkpoint for one sequence of `input_ids`."""
    import furiosa_opt_engine as engine

    from . import catalog

    comp = catalog.compose(engine.Checkpoint(directory))
    if comp.family != "mamba":
        raise ValueError(f"{comp.architecture}: not a Mamba model")
    with open(os.path.join(directory, "config.json")) as f:
        cfg = json.load(f)
    t = load_tensors(directory)
    eps = float(cfg.get("layer_norm_epsilon", 1e-5))
    ids = input_ids.long().view(-1)
    n = ids.numel()
    x = t["backbone.embeddings.weight"][ids]
    for layer in range(int(cfg["num_hidden_layers"])):
        p = f"backbone.layers.{layer}."
        m = p + "mixer."
        h = _rms(x, t[p + "norm.weight"], eps)
        proj = h @ t[m + "in_proj.weight"].T
        if m + "in_proj.bias" in t:
            proj = proj + t[m + "in_proj.bias"]
        xs, z = proj.chunk(2, dim=-1)
        xs = _causal_conv(xs, t[m + "conv1d.weight"][:, 0, :], t.get(m + "conv1d.bias"))
        a = -torch.exp(t[m + "A_log"])  # [inner, state]
        state = a.shape[1]
        rank = t[m + "dt_proj.weight"].shape[1]
        dbc = xs @ t[m + "x_proj.weight"].T
        dt, b, c = dbc.split([rank, state, state], dim=-1)
        dt = torch.nn.functional.softplus(dt @ t[m + "dt_proj.weight"].T + t[m + "dt_proj.bias"])  # [n, inner]
        s = torch.zeros_like(a)
        ys = []
        for i in range(n):
            s = torch.exp(dt[i][:, None] * a) * s + (dt[i] * xs[i])[:, None] * b[i][None, :]
            ys.append(s @ c[i] + t[m + "D"] * xs[i])
        y = torch.stack(ys) * torch.nn.functional.silu(z)
        out = y @ t[m + "out_proj.weight"].T
        if m + "out_proj.bias" in t:
            out = out + t[m + "out_proj.bias"]
        x = x + out
    x = _rms(x, t["backbone.norm_f.weight"], eps)
    return x @ t.get("lm_head.weight", t["backbone.embeddings.weight"]).T


def _mamba2_mixer(t, m, h, inner, heads, groups, state, eps, lo, hi):
    """A Mamba-2 mixer (names under `m`) over normed rows h [n, d]: in_proj to z, x, B, C and dt, a
    causal depthwise convolution and SiLU over x, B, C, the scan as its recurrence, the gated
    RMSNorm and out_proj."""
    n = h.shape[0]
    head_dim = inner // heads
    proj = h @ t[m + "in_proj.weight"].T
    if m + "in_proj.bias" in t:
        proj = proj + t[m + "in_proj.bias"]
    conv_dim = inner + 2 * groups * state
    z, xbc, dt = proj.split([inner, conv_dim, heads], dim=-1)
    conv = _causal_conv(xbc, t[m + "conv1d.weight"][:, 0, :], t.get(m + "conv1d.bias"))
    xs, bs, cs = conv.split([inner, groups * state, groups * state], dim=-1)
    dt = torch.nn.functional.softplus(dt + t[m + "dt_bias"]).clamp(lo, hi)  # [n, heads]
    a = -torch.exp(t[m + "A_log"])
    s = torch.zeros(heads, head_dim, state)
    ys = []
    per = heads // groups
    for i in range(n):
        xh = xs[i].view(heads, head_dim)
        b = bs[i].view(groups, state).repeat_interleave(per, dim=0)  # [heads, state]
        c = cs[i].view(groups, state).repeat_interleave(per, dim=0)
        s = s * torch.exp(dt[i] * a)[:, None, None] + (dt[i][:, None] * xh)[:, :, None] * b[:, None, :]
        ys.append((s @ c[:, :, None])[..., 0] + t[m + "D"][:, None] * xh)
    y = torch.stack(ys).reshape(n, inner)
    y = _rms(y * torch.nn.functional.silu(z), t[m + "norm.weight"], eps)
    out = y @ t[m + "out_proj.weight"].T
    if m + "out_proj.bias" in t:
        out = out + t[m + "out_proj.bias"]
    return out


def _step_limit(cfg) -> tuple[float, float]:
    """The clamp of a Mamba-2 mixer's dt (`time_step_limit`, unbounded by default)."""
    lo, hi = cfg.get("time_step_limit") or (0.0, float("inf"))
    lo = float(lo) if isinstance(lo, (int, float)) else 0.0
    hi = float(hi) if isinstance(hi, (int, float)) else float("inf")
    return lo, hi


def _rotate(x: torch.Tensor, theta: float, rot: int) -> torch.Tensor:
    """RoPE (rotate-half pairing) of the first `rot` dims of x [n, heads, head], positions 0..n-1."""
    inv = 1.0 / theta ** (torch.arange(0, rot, 2).float() / rot)
    ang = torch.arange(x.shape[0]).float()[:, None] * inv[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], -1)[:, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], -1)[:, None, :]
    xr, xp = x[..., :rot], x[..., rot:]
    half = torch.cat([-xr[..., rot // 2 :], xr[..., : rot // 2]], -1)
    return torch.cat([xr * cos + half * sin, xp], -1)


def bamba(directory: str, input_ids: torch.Tensor) -> torch.Tensor:
    """Logits [tokens, vocab] of a Bamba checkpoint for one sequence of `input_ids`."""
    import furiosa_opt_engine as engine

    from . import catalog

    comp = catalog.compose(engine.Checkpoint(directory))
    if comp.family != "bamba":
        raise ValueError(f"{comp.architecture}: not a Bamba model")
    with open(os.path.join(directory, "config.json")) as f:
        cfg = json.load(f)
    t = load_tensors(directory)
    d = int(cfg["hidden_size"])
    heads = int(cfg["num_attention_heads"])
    kv = int(cfg.get("num_key_value_heads", heads))
    hd = d // heads
    inner = int(cfg.get("mamba_expand", 2)) * d
    eps = float(cfg.get("rms_norm_eps", 1e-5))
    rope = cfg.get("rope_parameters") or {}
    theta = float(rope.get("rope_theta", cfg.get("rope_theta", 10000.0)))
    # The rotated prefix of each head: `attn_rotary_emb` dims (the original Bamba config key), else
    # head_dim x partial_rotary_factor (the top-level key, else the one in rope_parameters).
    factor = cfg.get("partial_rotary_factor", rope.get("partial_rotary_factor", 0.5))
    rot = int(cfg.get("attn_rotary_emb") or hd * float(factor))
    attention = set(cfg.get("attn_layer_indices") or [])
    lo, hi = _step_limit(cfg)
    ids = input_ids.long().view(-1)
    n = ids.numel()
    x = t["model.embed_tokens.weight"][ids]
    causal = torch.triu(torch.full((n, n), float("-inf")), 1)
    for layer in range(int(cfg["num_hidden_layers"])):
        p = f"model.layers.{layer}."
        h = _rms(x, t[p + "input_layernorm.weight"], eps)
        if layer in attention:
            q = _rotate((h @ t[p + "self_attn.q_proj.weight"].T).view(n, heads, hd), theta, rot)
            k = _rotate((h @ t[p + "self_attn.k_proj.weight"].T).view(n, kv, hd), theta, rot)
            v = (h @ t[p + "self_attn.v_proj.weight"].T).view(n, kv, hd)
            k, v = (z.repeat_interleave(heads // kv, dim=1) for z in (k, v))
            att = torch.softmax(torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(hd) + causal, dim=-1)
            out = torch.einsum("hqk,khd->qhd", att, v).reshape(n, heads * hd) @ t[p + "self_attn.o_proj.weight"].T
        else:
            out = _mamba2_mixer(t, p + "mamba.", h, inner, int(cfg["mamba_n_heads"]), int(cfg.get("mamba_n_groups", 1)),
                                int(cfg.get("mamba_d_state", 256)), eps, lo, hi)
        x = x + out
        h = _rms(x, t[p + "pre_ff_layernorm.weight"], eps)
        f = p + "feed_forward."
        x = x + (torch.nn.functional.silu(h @ t[f + "gate_proj.weight"].T) * (h @ t[f + "up_proj.weight"].T)) @ \
            t[f + "down_proj.weight"].T
    x = _rms(x, t["model.final_layernorm.weight"], eps)
    return x @ t.get("lm_head.weight", t["model.embed_tokens.weight"]).T


def gemma3(directory: str, input_ids: torch.Tensor) -> torch.Tensor:
    """Logits [tokens, vocab] of a Gemma-3 text checkpoint for one sequence of `input_ids`."""
    import furiosa_opt_engine as engine

    from . import catalog

    comp = catalog.compose(engine.Checkpoint(directory))
    if comp.family != "gemma3_text":
        raise ValueError(f"{comp.architecture}: not a Gemma-3 text model")
    with open(os.path.join(directory, "config.json")) as f:
        cfg = json.load(f)
    t = load_tensors(directory)
    d, L = int(cfg["hidden_size"]), int(cfg["num_hidden_layers"])
    heads = int(cfg["num_attention_heads"])
    kv = int(cfg.get("num_key_value_heads", heads))
    hd = int(cfg.get("head_dim", 256))
    eps = float(cfg.get("rms_norm_eps", 1e-6))
    window = int(cfg.get("sliding_window", 4096))
    scale = float(cfg.get("query_pre_attn_scalar", hd)) ** -0.5
    rope = cfg.get("rope_parameters") or {}
    theta = {"full_attention": float((rope.get("full_attention") or {}).get("rope_theta", cfg.get("rope_theta", 1e6))),
             "sliding_attention": float((rope.get("sliding_attention") or {}).get(
                 "rope_theta", cfg.get("rope_local_base_freq", 1e4)))}
    types = cfg.get("layer_types") or ["full_attention" if (i + 1) % int(cfg.get("sliding_window_pattern", 6)) == 0
                                       else "sliding_attention" for i in range(L)]

    def norm(x, w):
        return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)) * (1.0 + w)

    ids = input_ids.long().view(-1)
    n = ids.numel()
    x = t["model.embed_tokens.weight"][ids] * torch.tensor(d ** 0.5)
    i, j = torch.arange(n)[:, None], torch.arange(n)[None, :]
    masks = {"full_attention": torch.where(j <= i, 0.0, float("-inf")),
             "sliding_attention": torch.where((j <= i) & (j > i - window), 0.0, float("-inf"))}
    for layer in range(L):
        p = f"model.layers.{layer}."
        kind = types[layer]
        h = norm(x, t[p + "input_layernorm.weight"])
        q = norm((h @ t[p + "self_attn.q_proj.weight"].T).view(n, heads, hd), t[p + "self_attn.q_norm.weight"])
        k = norm((h @ t[p + "self_attn.k_proj.weight"].T).view(n, kv, hd), t[p + "self_attn.k_norm.weight"])
        v = (h @ t[p + "self_attn.v_proj.weight"].T).view(n, kv, hd)
        q, k = _rotate(q, theta[kind], hd), _rotate(k, theta[kind], hd)
        k, v = (z.repeat_interleave(heads // kv, dim=1) for z in (k, v))
        att = torch.softmax(torch.einsum("qhd,khd->hqk", q, k) * scale + masks[kind], dim=-1)
        out = torch.einsum("hqk,khd->qhd", att, v).reshape(n, heads * hd) @ t[p + "self_attn.o_proj.weight"].T
        x = x + norm(out, t[p + "post_attention_layernorm.weight"])
        h = norm(x, t[p + "pre_feedforward_layernorm.weight"])
        mid = torch.nn.functional.gelu(h @ t[p + "mlp.gate_proj.weight"].T, approximate="tanh") * (h @ t[p + "mlp.up_proj.weight"].T)
        x = x + norm(mid @ t[p + "mlp.down_proj.weight"].T, t[p + "post_feedforward_layernorm.weight"])
    x = norm(x, t["model.norm.weight"])
    logits = x @ t.get("lm_head.weight", t["model.embed_tokens.weight"]).T
    cap = cfg.get("final_logit_softcapping")
    return logits if not cap else torch.tanh(logits / cap) * cap


def _rotate_freqs(x: torch.Tensor, inv: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE of x [n, heads, head] with the inverse frequencies `inv` [head / 2]
    (zeros leave their pairs unrotated), positions 0..n-1."""
    ang = torch.arange(x.shape[0]).float()[:, None] * inv[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], -1)[:, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], -1)[:, None, :]
    h = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., h:], x[..., :h]], -1) * sin


def _inv_freq(params: dict, head: int) -> torch.Tensor:
    theta = float(params.get("rope_theta", 10000.0))
    if params.get("rope_type", "default") == "proportional":
        # Only the first partial_rotary_factor of the head's frequencies turn, at the whole head's
        # spacing; the other pairs keep frequency zero.
        turning = int(head * float(params.get("partial_rotary_factor", 1.0))) // 2
        inv = torch.zeros(head // 2)
        inv[:turning] = 1.0 / theta ** (torch.arange(0, 2 * turning, 2).float() / head)
        return inv
    return 1.0 / theta ** (torch.arange(0, head, 2).float() / head)


def gemma4(directory: str, input_ids: torch.Tensor) -> torch.Tensor:
    """Logits [tokens, vocab] of a Gemma-4 text checkpoint for one sequence of `input_ids`."""
    import furiosa_opt_engine as engine

    from . import catalog

    comp = catalog.compose(engine.Checkpoint(directory))
    if comp.family != "gemma4_text":
        raise ValueError(f"{comp.architecture}: not a Gemma-4 text model")
    with open(os.path.join(directory, "config.json")) as f:
        cfg = json.load(f)
    if cfg.get("enable_moe_block"):
        raise NotImplementedError("enable_moe_block: the host forward does not cover the expert block")
    t = load_tensors(directory)
    d, L = int(cfg["hidden_size"]), int(cfg["num_hidden_layers"])
    heads = int(cfg["num_attention_heads"])
    kv = int(cfg.get("num_key_value_heads", heads))
    hd = int(cfg.get("head_dim", 256))
    ghd = int(cfg.get("global_head_dim") or hd)
    gkv = int(cfg.get("num_global_key_value_heads") or kv)
    eps = float(cfg.get("rms_norm_eps", 1e-6))
    window = int(cfg.get("sliding_window", 512))
    k_eq_v = bool(cfg.get("attention_k_eq_v"))
    ple = int(cfg.get("hidden_size_per_layer_input") or 0)
    rope = cfg.get("rope_parameters") or {}
    types = cfg["layer_types"]

    def norm(x, w=None):
        y = x * (x.pow(2).mean(-1, keepdim=True) + eps) ** -0.5
        return y if w is None else y * w

    ids = input_ids.long().view(-1)
    n = ids.numel()
    x = t["model.embed_tokens.weight"][ids] * torch.tensor(d ** 0.5)
    if ple:
        per = t["model.embed_tokens_per_layer.weight"][ids].view(n, L, ple) * torch.tensor(ple ** 0.5)
        proj = (x @ t["model.per_layer_model_projection.weight"].T * d ** -0.5).view(n, L, ple)
        per = (norm(proj, t["model.per_layer_projection_norm.weight"]) + per) * 2 ** -0.5
    i, j = torch.arange(n)[:, None], torch.arange(n)[None, :]
    masks = {"full_attention": torch.where(j <= i, 0.0, float("-inf")),
             "sliding_attention": torch.where((j <= i) & (j > i - window), 0.0, float("-inf"))}
    for layer in range(L):
        p = f"model.layers.{layer}."
        kind = types[layer]
        full = kind == "full_attention"
        h_dim = ghd if full else hd
        nkv = gkv if (k_eq_v and full) else kv
        inv = _inv_freq(rope.get(kind, {}), h_dim)
        h = norm(x, t[p + "input_layernorm.weight"])
        q = _rotate_freqs(norm((h @ t[p + "self_attn.q_proj.weight"].T).view(n, heads, h_dim),
                               t[p + "self_attn.q_norm.weight"]), inv)
        k_raw = (h @ t[p + "self_attn.k_proj.weight"].T).view(n, nkv, h_dim)
        v_raw = k_raw if (k_eq_v and full) else (h @ t[p + "self_attn.v_proj.weight"].T).view(n, nkv, h_dim)
        k = _rotate_freqs(norm(k_raw, t[p + "self_attn.k_norm.weight"]), inv)
        v = norm(v_raw)
        k, v = (z.repeat_interleave(heads // nkv, dim=1) for z in (k, v))
        att = torch.softmax(torch.einsum("qhd,khd->hqk", q, k) + masks[kind], dim=-1)
        out = torch.einsum("hqk,khd->qhd", att, v).reshape(n, heads * h_dim) @ t[p + "self_attn.o_proj.weight"].T
        x = x + norm(out, t[p + "post_attention_layernorm.weight"])
        h = norm(x, t[p + "pre_feedforward_layernorm.weight"])
        mid = torch.nn.functional.gelu(h @ t[p + "mlp.gate_proj.weight"].T, approximate="tanh") * (h @ t[p + "mlp.up_proj.weight"].T)
        x = x + norm(mid @ t[p + "mlp.down_proj.weight"].T, t[p + "post_feedforward_layernorm.weight"])
        if ple:
            g = torch.nn.functional.gelu(x @ t[p + "per_layer_input_gate.weight"].T, approximate="tanh") * per[:, layer]
            x = x + norm(g @ t[p + "per_layer_projection.weight"].T, t[p + "post_per_layer_input_norm.weight"])
        x = x * t[p + "layer_scalar"]
    x = norm(x, t["model.norm.weight"])
    logits = x @ t.get("lm_head.weight", t["model.embed_tokens.weight"]).T
    cap = cfg.get("final_logit_softcapping")
    return logits if not cap else torch.tanh(logits / cap) * cap


def olmoe(directory: str, input_ids: torch.Tensor) -> torch.Tensor:
    """Logits [tokens, vocab] of an OLMoE checkpoint for one sequence of `input_ids`."""
    import furiosa_opt_engine as engine

    from . import catalog

    comp = catalog.compose(engine.Checkpoint(directory))
    if comp.family != "olmoe":
        raise ValueError(f"{comp.architecture}: not an OLMoE model")
    with open(os.path.join(directory, "config.json")) as f:
        cfg = json.load(f)
    t = load_tensors(directory)
    d, L = int(cfg["hidden_size"]), int(cfg["num_hidden_layers"])
    heads = int(cfg["num_attention_heads"])
    kv = int(cfg.get("num_key_value_heads", heads))
    hd = d // heads
    eps = float(cfg.get("rms_norm_eps", 1e-5))
    experts, top = int(cfg["num_experts"]), int(cfg.get("num_experts_per_tok", 8))
    theta = float((cfg.get("rope_parameters") or {}).get("rope_theta", cfg.get("rope_theta", 10000.0)))
    inv = 1.0 / theta ** (torch.arange(0, hd, 2).float() / hd)
    ids = input_ids.long().view(-1)
    n = ids.numel()
    x = t["model.embed_tokens.weight"][ids]
    causal = torch.triu(torch.full((n, n), float("-inf")), 1)
    for layer in range(L):
        p = f"model.layers.{layer}."
        h = _rms(x, t[p + "input_layernorm.weight"], eps)
        q = _rms(h @ t[p + "self_attn.q_proj.weight"].T, t[p + "self_attn.q_norm.weight"], eps).view(n, heads, hd)
        k = _rms(h @ t[p + "self_attn.k_proj.weight"].T, t[p + "self_attn.k_norm.weight"], eps).view(n, kv, hd)
        v = (h @ t[p + "self_attn.v_proj.weight"].T).view(n, kv, hd)
        q, k = _rotate_freqs(q, inv), _rotate_freqs(k, inv)
        k, v = (z.repeat_interleave(heads // kv, dim=1) for z in (k, v))
        att = torch.softmax(torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(hd) + causal, dim=-1)
        x = x + torch.einsum("hqk,khd->qhd", att, v).reshape(n, d) @ t[p + "self_attn.o_proj.weight"].T
        h = _rms(x, t[p + "post_attention_layernorm.weight"], eps)
        probs = torch.softmax(h @ t[p + "mlp.gate.weight"].T, dim=-1)
        weights, chosen = probs.topk(top, dim=-1)
        if cfg.get("norm_topk_prob"):
            weights = weights / weights.sum(-1, keepdim=True)
        out = torch.zeros_like(x)
        for e in range(experts):
            rows, slot = (chosen == e).nonzero(as_tuple=True)
            if rows.numel() == 0:
                continue
            q_ = f"{p}mlp.experts.{e}."
            he = h[rows]
            y = (torch.nn.functional.silu(he @ t[q_ + "gate_proj.weight"].T) * (he @ t[q_ + "up_proj.weight"].T)) @ \
                t[q_ + "down_proj.weight"].T
            out.index_add_(0, rows, y * weights[rows, slot][:, None])
        x = x + out
    x = _rms(x, t["model.norm.weight"], eps)
    return x @ t.get("lm_head.weight", t["model.embed_tokens.weight"]).T


def _rotate_pairs(x: torch.Tensor, inv: torch.Tensor) -> torch.Tensor:
    """RoPE on adjacent pairs (2i, 2i + 1) of x [n, heads, dims], positions 0..n-1."""
    ang = torch.arange(x.shape[0]).float()[:, None] * inv[None, :]
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
    a, b = x[..., 0::2], x[..., 1::2]
    return torch.stack([a * cos - b * sin, a * sin + b * cos], dim=-1).flatten(-2)


def deepseek_v2(directory: str, input_ids: torch.Tensor) -> torch.Tensor:
    """Logits [tokens, vocab] of a DeepSeek-V2 checkpoint for one sequence of `input_ids`."""
    import furiosa_opt_engine as engine

    from . import catalog

    comp = catalog.compose(engine.Checkpoint(directory))
    if comp.family != "deepseek_v2":
        raise ValueError(f"{comp.architecture}: not a DeepSeek-V2 model")
    with open(os.path.join(directory, "config.json")) as f:
        cfg = json.load(f)
    t = load_tensors(directory)
    L, heads = int(cfg["num_hidden_layers"]), int(cfg["num_attention_heads"])
    nope, rope_d, vd = int(cfg["qk_nope_head_dim"]), int(cfg["qk_rope_head_dim"]), int(cfg["v_head_dim"])
    kv_rank = int(cfg["kv_lora_rank"])
    eps = float(cfg.get("rms_norm_eps", 1e-6))
    experts, top = int(cfg.get("n_routed_experts") or 0), int(cfg.get("num_experts_per_tok") or 0)
    dense, freq = int(cfg.get("first_k_dense_replace") or 0), int(cfg.get("moe_layer_freq") or 1)
    scale_out = float(cfg.get("routed_scaling_factor") or 1.0)
    method = cfg.get("topk_method") or "greedy"
    theta = float((cfg.get("rope_parameters") or {}).get("rope_theta", cfg.get("rope_theta", 10000.0)))
    inv = 1.0 / theta ** (torch.arange(0, rope_d, 2).float() / rope_d)
    ids = input_ids.long().view(-1)
    n = ids.numel()
    x = t["model.embed_tokens.weight"][ids]
    causal = torch.triu(torch.full((n, n), float("-inf")), 1)

    def mlp(prefix, h):
        return (torch.nn.functional.silu(h @ t[prefix + "gate_proj.weight"].T) * (h @ t[prefix + "up_proj.weight"].T)) @ \
            t[prefix + "down_proj.weight"].T

    for layer in range(L):
        p = f"model.layers.{layer}."
        a = p + "self_attn."
        h = _rms(x, t[p + "input_layernorm.weight"], eps)
        if a + "q_a_proj.weight" in t:
            q = _rms(h @ t[a + "q_a_proj.weight"].T, t[a + "q_a_layernorm.weight"], eps) @ t[a + "q_b_proj.weight"].T
        else:
            q = h @ t[a + "q_proj.weight"].T
        q = q.view(n, heads, nope + rope_d)
        q_nope, q_pe = q.split([nope, rope_d], dim=-1)
        ckv = h @ t[a + "kv_a_proj_with_mqa.weight"].T
        latent, k_pe = ckv.split([kv_rank, rope_d], dim=-1)
        kvb = (_rms(latent, t[a + "kv_a_layernorm.weight"], eps) @ t[a + "kv_b_proj.weight"].T).view(n, heads, nope + vd)
        k_nope, v = kvb.split([nope, vd], dim=-1)
        q_pe = _rotate_pairs(q_pe, inv)
        k_pe = _rotate_pairs(k_pe.view(n, 1, rope_d), inv).expand(n, heads, rope_d)
        qs, ks = torch.cat([q_nope, q_pe], -1), torch.cat([k_nope, k_pe], -1)
        att = torch.softmax(torch.einsum("qhd,khd->hqk", qs, ks) / math.sqrt(nope + rope_d) + causal, dim=-1)
        x = x + torch.einsum("hqk,khd->qhd", att, v).reshape(n, heads * vd) @ t[a + "o_proj.weight"].T
        h = _rms(x, t[p + "post_attention_layernorm.weight"], eps)
        if experts and layer >= dense and layer % freq == 0:
            probs = torch.softmax(h @ t[p + "mlp.gate.weight"].T, dim=-1)
            if method == "group_limited_greedy":
                groups, keep = int(cfg["n_group"]), int(cfg["topk_group"])
                best = probs.view(n, groups, -1).max(-1).values.topk(keep, dim=-1).indices
                allowed = torch.zeros(n, groups).scatter_(1, best, 1.0).repeat_interleave(experts // groups, dim=1)
                probs_masked = probs.masked_fill(allowed == 0, 0.0)
                weights, chosen = probs_masked.topk(top, dim=-1)
            else:
                weights, chosen = probs.topk(top, dim=-1)
            weights = weights * scale_out
            out = torch.zeros_like(x)
            for e in range(experts):
                rows, slot = (chosen == e).nonzero(as_tuple=True)
                if rows.numel():
                    out.index_add_(0, rows, mlp(f"{p}mlp.experts.{e}.", h[rows]) * weights[rows, slot][:, None])
            if p + "mlp.shared_experts.gate_proj.weight" in t:
                out = out + mlp(p + "mlp.shared_experts.", h)
            x = x + out
        else:
            x = x + mlp(p + "mlp.", h)
    x = _rms(x, t["model.norm.weight"], eps)
    return x @ t.get("lm_head.weight", t["model.embed_tokens.weight"]).T
