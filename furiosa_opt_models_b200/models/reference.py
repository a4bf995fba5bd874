"""Plain PyTorch FP32 math of the decoder ops: the oracle every kernel and the engine's CPU path
are checked against.

Each function states the numerical contract of the reference op it restates:
RMSNorm (`ops/normalization/rms_norm.rs:15-20`), RoPE with half-split pairs (`ops/rotary.rs:55-57`),
SwiGLU with SiLU(gate) rounded before the product (`ops/swiglu/mod.rs:1-3`).
"""

from __future__ import annotations

import torch


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """FP32 statistics, FP32 product with the weight, no intermediate rounding."""
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()


def rope(x: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor, factor: float = 1.0) -> torch.Tensor:
    """Rotates pairs (j, j + d/2) of the last axis by ``position * inv_freq[j]``.

    ``x`` is [rows, heads, d] and ``positions`` [rows]."""
    angle = positions.float()[:, None] * inv_freq.float()[None, :]
    cos = (torch.cos(angle) * factor)[:, None, :]
    sin = (torch.sin(angle) * factor)[:, None, :]
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def qk_front(qkv, q_heads, kv_heads, head_dim, q_norm, k_norm, eps, positions, inv_freq, factor=1.0,
             round_bf16=True):
    """Splits packed q/k/v rows, applies the per-head norm and RoPE to q and k.

    With ``round_bf16`` the norm's output is rounded to BF16 before the rotation, as the kernel
    stores it."""
    rows = qkv.shape[0]
    q = qkv[:, : q_heads * head_dim].reshape(rows, q_heads, head_dim).float()
    k = qkv[:, q_heads * head_dim : (q_heads + kv_heads) * head_dim].reshape(rows, kv_heads, head_dim).float()
    v = qkv[:, (q_heads + kv_heads) * head_dim :].reshape(rows, kv_heads, head_dim).float()
    if q_norm is not None:
        q = rmsnorm(q, q_norm, eps)
        k = rmsnorm(k, k_norm, eps)
        if round_bf16:
            q = q.bfloat16().float()
            k = k.bfloat16().float()
    return rope(q, positions, inv_freq, factor), rope(k, positions, inv_freq, factor), v


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``bf16(silu(bf16 gate)) * bf16 up`` in FP32."""
    g = gate.bfloat16().float()
    return torch.nn.functional.silu(g).bfloat16().float() * up.bfloat16().float()


def gather_kv(cache: torch.Tensor, table, table_start: int, keys: int):
    """K and V [keys, kv_heads, d] of one sequence from a paged layer ``cache``
    [blocks, 2, kv_heads, 16, d]."""
    nb = (keys + 15) // 16
    ids = [int(x) for x in table[table_start : table_start + nb]]
    pages = cache[ids]  # [nb, 2, H, 16, d]
    k = pages[:, 0].permute(0, 2, 1, 3).reshape(nb * 16, cache.shape[2], cache.shape[4])[:keys]
    v = pages[:, 1].permute(0, 2, 1, 3).reshape(nb * 16, cache.shape[2], cache.shape[4])[:keys]
    return k.float(), v.float()


def paged_attention(q: torch.Tensor, cache: torch.Tensor, table, segments, scale: float | None = None,
                    causal: bool = True):
    """GQA attention of every segment's rows over its paged history, in FP32.

    ``q`` [rows, q_heads, d]; ``segments`` rows of (row_start, len, cached, table_start, nblocks).
    Row i of a segment is position cached + i and attends keys 0..cached + i (causal), or every
    key 0..cached + len - 1 of its segment (``causal=False``)."""
    rows, q_heads, d = q.shape
    kv_heads = cache.shape[2]
    group = q_heads // kv_heads
    scale = d ** -0.5 if scale is None else scale
    out = torch.zeros(rows, q_heads, d, dtype=torch.float32)
    for row_start, length, cached, table_start, _ in [tuple(int(x) for x in s) for s in segments]:
        keys = cached + length
        k, v = gather_kv(cache, table, table_start, keys)
        k = k.repeat_interleave(group, dim=1)  # [keys, q_heads, d]
        v = v.repeat_interleave(group, dim=1)
        qs = q[row_start : row_start + length].float()  # [len, q_heads, d]
        s = torch.einsum("lhd,khd->hlk", qs, k) * scale
        pos = torch.arange(length)[:, None] + cached
        mask = torch.arange(keys)[None, :] <= (pos if causal else torch.full_like(pos, keys - 1))
        s = s.masked_fill(~mask[None], float("-inf"))
        out[row_start : row_start + length] = torch.einsum("hlk,khd->lhd", torch.softmax(s, -1), v)
    return out


# ------------------------------------------------------------------------------ quantized weights
# FP8 block contract: E4M3 codes, one FP32 scale per 128 x 128 block, a group's scale its largest
# magnitude over 448 and never below 1e-10 (crates/furiosa-opt-models/src/tensor/form/fp8.rs:1-12).
# NVFP4: E2M1 codes, an E4M3 scale per 16 inputs, an FP32 tensor scale multiplying the reduced sum
# ("Late", crates/furiosa-opt-models/src/tensor/form/nvfp4.rs:1-10).

E4M3_MAX = 448.0
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def _e4m3(x: torch.Tensor) -> torch.Tensor:
    """E4M3 bytes of FP32 values, rounded to nearest even and saturated at +-448."""
    return x.clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)


def _e4m3_value(b: torch.Tensor) -> torch.Tensor:
    return b.view(torch.float8_e4m3fn).float()


def fp8_block_quantize(w: torch.Tensor):
    """BF16 [rows, cols] -> (E4M3 codes uint8 [rows, cols], FP32 scales [rows/128, cols/128])."""
    rows, cols = w.shape
    br, bc = (rows + 127) // 128, (cols + 127) // 128
    wf = torch.zeros(br * 128, bc * 128, dtype=torch.float32, device=w.device)
    wf[:rows, :cols] = w.float()
    amax = wf.view(br, 128, bc, 128).abs().amax(dim=(1, 3))
    # Tensor-by-tensor divisions: PyTorch divides by a Python scalar as a product with its
    # reciprocal on CUDA, which is not the correctly rounded quotient the kernels compute.
    scales = torch.clamp(amax, min=1e-10) * torch.full_like(amax, 1.0 / E4M3_MAX)
    s = scales.repeat_interleave(128, 0).repeat_interleave(128, 1)[:rows, :cols]
    return _e4m3(w.float() / s), scales


def fp8_quantize_input(x: torch.Tensor):
    """W8A8 inputs per (row, 128-input group): scale = max(amax, 1e-10) * fl(1/448), codes
    e4m3_sat(x / scale) -> (codes uint8 [rows, K], FP32 scales [rows, K/128])."""
    rows, K = x.shape
    xf = x.float().view(rows, K // 128, 128)
    amax = xf.abs().amax(-1)
    scales = torch.clamp(amax, min=1e-10) * torch.full_like(amax, 1.0 / E4M3_MAX)
    return _e4m3(xf / scales[..., None]).view(rows, K), scales


def fp8_block_w8a8(a: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """The FP8 block contract of one GEMM: each 128-input block's FP32 sum times its activation
    scale, then its weight scale, the blocks added in order -> FP32 [rows, out]."""
    ac, asc = fp8_quantize_input(a)
    av = _e4m3_value(ac)
    wv = _e4m3_value(codes)
    rows, K = ac.shape
    N = codes.shape[0]
    out = torch.zeros(rows, N, dtype=torch.float32, device=a.device)
    wsc = scales.repeat_interleave(128, 0)[:N]  # [N, K/128]
    for g in range(K // 128):
        part = av[:, g * 128:(g + 1) * 128] @ wv[:, g * 128:(g + 1) * 128].T
        out += (part * asc[:, g:g + 1]) * wsc[:, g][None, :]
    return out


def fp8_block_dequantize(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Each coefficient ``code * block scale``, rounded once to BF16, as FP32."""
    rows, cols = codes.shape
    s = scales.repeat_interleave(128, 0).repeat_interleave(128, 1)[:rows, :cols]
    return (_e4m3_value(codes) * s).bfloat16().float()


def _e2m1_code(x: torch.Tensor) -> torch.Tensor:
    """Nearest E2M1 code of each value, ties to the even code; the sign in bit 3."""
    vals = torch.tensor(E2M1_VALUES, dtype=torch.float32, device=x.device)
    d = (x.abs()[..., None] - vals).abs()
    tie = d == d.amin(-1, keepdim=True)
    idx = torch.arange(8, device=x.device)
    # Lowest index among the nearest, preferring an even one when two are equally near.
    key = torch.where(tie, idx + 16 * (idx % 2), torch.full_like(idx, 1 << 10))
    code = key.argmin(-1).to(torch.uint8)
    return code | ((x < 0).to(torch.uint8) << 3)


def _nvfp4_groups(x: torch.Tensor, glob: torch.Tensor):
    """E2M1 codes [rows, cols] (uint8, sign in bit 3) and E4M3 scale bytes [rows, cols/16] of FP32
    values under the tensor scale ``glob``: s = e4m3(amax/6 * glob), code = e2m1(x / (s * (1/glob)))."""
    rows, cols = x.shape
    blocks = x.view(rows, cols // 16, 16)
    bmax = blocks.abs().amax(-1)
    s8 = _e4m3((bmax / torch.full_like(bmax, 6.0)) * glob)
    restore = _e4m3_value(s8) * (torch.ones_like(glob) / glob)
    k = torch.where(restore != 0, torch.ones_like(restore) / restore, torch.zeros_like(restore))
    return _e2m1_code(blocks * k[..., None]).view(rows, cols), s8


def _pack_nibbles(codes: torch.Tensor) -> torch.Tensor:
    return codes[:, 0::2] | (codes[:, 1::2] << 4)


def nvfp4_quantize(w: torch.Tensor):
    """BF16 [rows, cols] -> (packed codes uint8 [rows, cols/2], E4M3 scales uint8 [rows, cols/16],
    FP32 tensor scale ``1 / global``), global = 448 * 6 / amax(W)."""
    wf = w.float()
    amax = wf.abs().max()
    glob = torch.full_like(amax, 448.0 * 6.0) / amax if amax > 0 else torch.ones_like(amax)
    codes, s8 = _nvfp4_groups(wf, glob)
    return _pack_nibbles(codes), s8, float(torch.ones_like(glob) / glob)


def nvfp4_quantize_input(x: torch.Tensor, input_scale: float):
    """W4A4 inputs: BF16 [rows, cols] under the fixed tensor scale ``global = 1 / input_scale``
    (FP32) -> (packed codes, E4M3 scales [rows, cols/16])."""
    glob = torch.ones((), dtype=torch.float32, device=x.device) / torch.tensor(
        input_scale, dtype=torch.float32, device=x.device)
    codes, s8 = _nvfp4_groups(x.float(), glob)
    return _pack_nibbles(codes), s8


def nvfp4_scale_atoms(s8: torch.Tensor) -> torch.Tensor:
    """Row-major scales [rows, K/16] -> 128-row-blocked atoms [ceil(rows/128), K/64, 512] in which
    the scale of (row r, group k) of a block sits at byte (r % 32) * 16 + (r / 32) * 4 + k."""
    rows, groups = s8.shape
    rb = (rows + 127) // 128
    padded = torch.zeros(rb * 128, groups, dtype=torch.uint8, device=s8.device)
    padded[:rows] = s8
    # [rb, r1 (4), r0 (32), kc, k (4)] -> [rb, kc, r0, r1, k]
    v = padded.view(rb, 4, 32, groups // 4, 4).permute(0, 3, 2, 1, 4)
    return v.reshape(rb, groups // 4, 512).contiguous()


def nvfp4_dequantize(packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """``code * block scale`` (exact in BF16) as FP32 [rows, cols]; the tensor scale is not applied."""
    rows = packed.shape[0]
    lo, hi = packed & 15, packed >> 4
    codes = torch.stack([lo, hi], dim=-1).view(rows, -1).long()
    vals = torch.tensor(E2M1_VALUES, dtype=torch.float32, device=packed.device)
    mag = vals[codes & 7]
    v = torch.where((codes & 8) != 0, -mag, mag)
    return v * _e4m3_value(scales).repeat_interleave(16, 1)


def nvfp4_scales_from_atoms(atoms: torch.Tensor, rows: int) -> torch.Tensor:
    """The inverse of ``nvfp4_scale_atoms``: row-major scales [rows, K/16]."""
    rb, kc, _ = atoms.shape
    v = atoms.view(rb, kc, 32, 4, 4).permute(0, 3, 2, 1, 4)  # [rb, r1, r0, kc, k]
    return v.reshape(rb * 128, kc * 4)[:rows].contiguous()


def quantized_linear(x: torch.Tensor, w) -> torch.Tensor:
    """``x @ W.T`` (FP32) under the contract of a quantized weight ``w`` (a ``QuantizedWeight``
    with codes and scales on any device): W8A8 for fp8_block, W4A4 for nvfp4_a4, W4A16 for nvfp4
    (``x`` is rounded to BF16 first, as the engine stores its inputs)."""
    dev = x.device
    codes, scales = w.codes.to(dev), w.scales.to(dev)
    xb = x.bfloat16()
    if w.format == "fp8_block":
        return fp8_block_w8a8(xb, codes, scales)
    if w.format == "fp8_block_w8a16":
        return xb.float() @ fp8_block_dequantize(codes, scales).T
    if w.format == "fp8_rows":
        return xb.float() @ (_e4m3_value(codes) * scales[:, None]).bfloat16().float().T
    if w.format == "nvfp4":
        return (xb.float() @ nvfp4_dequantize(codes, scales).T) * w.tensor_scale
    s8 = nvfp4_scales_from_atoms(scales, w.rows)
    ac, as8 = nvfp4_quantize_input(xb, w.input_scale)
    alpha = float(torch.tensor(w.input_scale, dtype=torch.float32) * torch.tensor(w.tensor_scale, dtype=torch.float32))
    return (nvfp4_dequantize(ac, as8) @ nvfp4_dequantize(codes, s8).T) * alpha


# ------------------------------------------------------------------------------ mixture of experts
# Routing and combine contract: crates/furiosa-opt-models/src/modules/feedforward/moe.rs:1-7
# (top-k of BF16 logits, best first, equal logits in ascending expert order; FP32 softmax; the
# weighted sum in FP32 in choice order, rounded once).


def moe_route(logits: torch.Tensor, k: int, normalize: bool = True):
    """(ids [rows, k] int64, weights [rows, k] FP32) of BF16 logits [rows, E]."""
    lf = logits.float()
    probs = torch.softmax(lf, dim=-1)
    rows, E = lf.shape
    # Stable descending sort keeps equal logits in ascending expert order.
    order = torch.sort(lf, dim=-1, descending=True, stable=True).indices[:, :k]
    w = torch.gather(probs, 1, order)
    if normalize:
        total = torch.zeros(rows, dtype=torch.float32, device=lf.device)
        for j in range(k):
            total = total + w[:, j]
        w = w / total[:, None]
    return order, w


def moe_forward(h: torch.Tensor, router: torch.Tensor, gate_up: torch.Tensor, down: torch.Tensor, k: int,
                normalize: bool = True):
    """The MoE block of BF16 rows h [T, H] -> BF16 [T, H]: router [E, H], gate_up [E, 2I, H] (128-row
    blocks alternating gate/up), down [E, H, I]. Router logits, expert rows and the output round to
    BF16 once each."""
    logits = (h.float() @ router.float().T).bfloat16()
    ids, w = moe_route(logits, k, normalize)
    T, H = h.shape
    acc = torch.zeros(T, H, dtype=torch.float32, device=h.device)
    for j in range(k):
        rows = torch.zeros(T, H, dtype=torch.float32, device=h.device)
        for e in ids[:, j].unique().tolist():
            sel = ids[:, j] == e
            gu = h[sel].float() @ gate_up[e].float().T
            blocks = gu.view(gu.shape[0], -1, 2, 128)
            g = blocks[:, :, 0].reshape(gu.shape[0], -1)
            u = blocks[:, :, 1].reshape(gu.shape[0], -1)
            act = swiglu(g, u).bfloat16().float()
            rows[sel] = (act @ down[e].float().T).bfloat16().float()
        acc = acc + w[:, j:j + 1] * rows
    return acc.bfloat16()


def fp8_rows_quantize(w: torch.Tensor, tensor_amax: float | None = None):
    """Load-time FP8 (crates/furiosa-opt-models/src/tensor/form/fp8.rs:195-220): scale =
    amax / 448 per row (or the tensor's), code = e4m3_sat(w * (1 / scale)), zero codes for a zero
    scale -> (codes uint8 [rows, cols], FP32 scales [rows])."""
    wf = w.float()
    amax = wf.abs().amax(-1) if tensor_amax is None else torch.full((w.shape[0],), float(tensor_amax), device=w.device)
    scales = amax / torch.full_like(amax, E4M3_MAX)
    rcp = torch.where(scales == 0, torch.zeros_like(scales), torch.ones_like(scales) / scales)
    return _e4m3(wf * rcp[:, None]), scales


# ------------------------------------------------------------------------------ media encoders
# Gemma-4 unified embedders (crates/furiosa-opt-models/src/models/vision_language/gemma4_unified.rs):
# every step rounded to BF16 as the BF16 forward rounds it.


def _bf(x: torch.Tensor) -> torch.Tensor:
    return x.bfloat16().float()


def _layernorm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    mean = x.mean(-1, keepdim=True)
    var = ((x - mean) ** 2).mean(-1, keepdim=True)
    return _bf((x - mean) * torch.rsqrt(var + eps) * w.float() + b.float())


def _unit_rms(x: torch.Tensor, eps: float) -> torch.Tensor:
    return _bf(x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps))


def gemma4_vision(w: dict, patches: torch.Tensor, positions, eps: float = 1e-6) -> torch.Tensor:
    """Rows [n, text] of merged patches [n, features] at (x, y) positions, in FP32 (BF16 values)."""
    e = "model.vision_embedder."
    x = _layernorm(patches.float(), w[e + "patch_ln1.weight"], w[e + "patch_ln1.bias"])
    v = _bf(x @ w[e + "patch_dense.weight"].float().T + w[e + "patch_dense.bias"].float())
    a = _layernorm(v, w[e + "patch_ln2.weight"], w[e + "patch_ln2.bias"])
    table = w[e + "pos_embedding"].float()
    xy = torch.tensor(positions, dtype=torch.long)
    pos = _bf(table[xy[:, 0], 0] + table[xy[:, 1], 1])
    s = _bf(a + pos)
    n = _layernorm(s, w[e + "pos_norm.weight"], w[e + "pos_norm.bias"])
    u = _unit_rms(n, eps)
    return _bf(u @ w["model.embed_vision.embedding_projection.weight"].float().T)


def gemma4_audio(w: dict, frames: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Rows [n, text] of audio frames [n, samples], in FP32 (BF16 values)."""
    u = _unit_rms(frames.float(), eps)
    return _bf(u @ w["model.embed_audio.embedding_projection.weight"].float().T)
