"""Torch-facing wrappers of the raw kernel launchers."""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .native import native, scratch

EPI_BF16, EPI_F32, EPI_SWIGLU = 0, 1, 2
MODE_AUTO, MODE_ROWS, MODE_SWAP = 0, 1, 2


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.data_ptr()


def _rowmajor(t: torch.Tensor, name: str) -> None:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D tensor with unit column stride")


W_BF16, W_FP8_W8A16, W_NVFP4, W_NVFP4_A4, W_FP8_BLOCK = 0, 1, 2, 3, 4


@dataclass
class QuantizedWeight:
    """A weight [rows, cols] held in a quantized format that the GEMM dequantizes on the fly.

    fp8_block: ``codes`` E4M3 as uint8 [rows, cols], ``scales`` FP32 [ceil(rows/128), ceil(cols/128)]
    (one per 128x128 block, the checkpoint's ``weight_scale_inv``); inputs quantize per 128-input
    group and each block's sum takes its scales (W8A8). fp8_block_w8a16: the same weights
    dequantized to BF16 in the kernel, BF16 inputs.
    fp8_rows: E4M3 ``codes`` [rows, cols] with one FP32 scale per row ``scales`` [rows] (FP8
    quantized at load per channel or per tensor), restored to BF16 in the kernel (W8A16).
    nvfp4: ``codes`` uint8 [rows, cols/2] (two E2M1 codes a byte, lower column in the low nibble),
    ``scales`` E4M3 as uint8 [rows, cols/16], ``tensor_scale`` the FP32 ``weight_scale_2``.
    nvfp4_a4 (W4A4 on the block-scaled MMA): ``codes`` as for nvfp4, ``scales`` the 128-row-blocked
    scale atoms [ceil(rows/128), cols/64, 512], ``input_scale`` the FP32 tensor scale the inputs
    quantize under; the sums take ``input_scale * tensor_scale``.
    """

    format: str
    codes: torch.Tensor
    scales: torch.Tensor
    rows: int
    cols: int
    tensor_scale: float = 1.0
    input_scale: float = 1.0
    # fp8_block on the W8A8 GEMM: the scales with each value four times (16-byte entries).
    gemm_scales: torch.Tensor | None = None

    def fp8_gemm_scales(self) -> torch.Tensor:
        if self.gemm_scales is None:
            s = self.scales.contiguous()
            self.gemm_scales = torch.empty(*s.shape, 4, dtype=torch.float32, device=s.device)
            native().ops.fp8_scales_pad4(s.data_ptr(), s.numel(), self.gemm_scales.data_ptr(), _stream())
        return self.gemm_scales

    @property
    def code(self) -> int:
        return {"fp8_block": W_FP8_BLOCK, "fp8_block_w8a16": W_FP8_W8A16, "fp8_rows": W_FP8_W8A16,
                "nvfp4": W_NVFP4, "nvfp4_a4": W_NVFP4_A4}[self.format]


def _f32(x: float) -> float:
    return float(torch.tensor(x, dtype=torch.float32))


def nvfp4_w4a4(q: QuantizedWeight, input_scale: float) -> QuantizedWeight:
    """The W4A4 form of an NVFP4 weight: its scales repacked into 128-row-blocked atoms."""
    if q.format != "nvfp4":
        raise ValueError("nvfp4_w4a4 takes an nvfp4 weight")
    if q.cols % 256:
        raise ValueError("W4A4 needs inputs in multiples of 256")
    atoms = torch.empty((q.rows + 127) // 128, q.cols // 64, 512, dtype=torch.uint8, device=q.codes.device)
    native().ops.nvfp4_scale_atoms(q.scales.data_ptr(), q.scales.stride(0), q.rows, q.cols,
                                   atoms.data_ptr(), _stream())
    return QuantizedWeight("nvfp4_a4", q.codes, atoms, q.rows, q.cols, q.tensor_scale, _f32(input_scale))


def quantize_nvfp4_input(x: torch.Tensor, input_scale: float):
    """W4A4 inputs: (packed codes [rows, K/2], scale atoms [ceil(rows/128), K/64, 512]) of BF16 ``x``
    under ``global = 1 / input_scale`` (FP32)."""
    _rowmajor(x, "x")
    rows, K = x.shape
    codes = torch.empty(rows, K // 2, dtype=torch.uint8, device=x.device)
    atoms = torch.empty((rows + 127) // 128, K // 64, 512, dtype=torch.uint8, device=x.device)
    glob = float(torch.tensor(1.0, dtype=torch.float32) / torch.tensor(input_scale, dtype=torch.float32))
    native().ops.quantize_nvfp4_act(x.data_ptr(), x.stride(0), rows, K, glob, codes.data_ptr(),
                                    codes.stride(0), atoms.data_ptr(), _stream())
    return codes, atoms


def quantize_fp8_input(x: torch.Tensor):
    """W8A8 inputs: (E4M3 codes uint8 [rows, K], FP32 scales [K/128, rows rounded up to 128])."""
    _rowmajor(x, "x")
    rows, K = x.shape
    pad = (rows + 127) // 128 * 128
    codes = torch.empty(rows, K, dtype=torch.uint8, device=x.device)
    scales = torch.empty(K // 128, pad, dtype=torch.float32, device=x.device)
    native().ops.quantize_fp8_act(x.data_ptr(), x.stride(0), rows, K, codes.data_ptr(), codes.stride(0),
                                  scales.data_ptr(), pad, _stream())
    return codes, scales


def quantize_fp8_rows(w: torch.Tensor, tensor_amax: float | None = None) -> QuantizedWeight:
    """FP8 of a BF16 weight with one scale per row (amax / 448), or per tensor with
    ``tensor_amax``; codes are ``w * (1 / scale)`` saturated."""
    _rowmajor(w, "w")
    w = w.contiguous()
    rows, cols = w.shape
    codes = torch.empty(rows, cols, dtype=torch.uint8, device=w.device)
    scales = torch.empty(rows, dtype=torch.float32, device=w.device)
    native().ops.quantize_fp8_rows(w.data_ptr(), rows, cols, -1.0 if tensor_amax is None else float(tensor_amax),
                                   codes.data_ptr(), scales.data_ptr(), _stream())
    return QuantizedWeight("fp8_rows", codes, scales, rows, cols)


def quantize_fp8_block(w: torch.Tensor) -> QuantizedWeight:
    """Block-scaled FP8 of a BF16 weight on the device (scale = max(amax, 1e-10) * fl(1/448))."""
    _rowmajor(w, "w")
    w = w.contiguous()
    rows, cols = w.shape
    codes = torch.empty(rows, cols, dtype=torch.uint8, device=w.device)
    scales = torch.empty((rows + 127) // 128, (cols + 127) // 128, dtype=torch.float32, device=w.device)
    native().ops.quantize_fp8_block(w.data_ptr(), rows, cols, codes.data_ptr(), scales.data_ptr(), _stream())
    return QuantizedWeight("fp8_block", codes, scales, rows, cols)


def quantize_nvfp4(w: torch.Tensor) -> QuantizedWeight:
    """NVFP4 of a BF16 weight on the device (global = 448 * 6 / amax; 16-column E4M3 scales)."""
    _rowmajor(w, "w")
    w = w.contiguous()
    rows, cols = w.shape
    if cols % 16:
        raise ValueError("NVFP4 needs columns in multiples of 16")
    codes = torch.empty(rows, cols // 2, dtype=torch.uint8, device=w.device)
    scales = torch.empty(rows, cols // 16, dtype=torch.uint8, device=w.device)
    amax = torch.zeros(2, dtype=torch.float32, device=w.device)
    ops = native().ops
    ops.absmax(w.data_ptr(), w.numel(), amax.data_ptr(), _stream())
    ops.quantize_nvfp4(w.data_ptr(), rows, cols, codes.data_ptr(), scales.data_ptr(), amax.data_ptr(),
                       amax.data_ptr() + 4, _stream())
    return QuantizedWeight("nvfp4", codes, scales, rows, cols, float(amax[1].item()))


def gemm(
    a: torch.Tensor,
    w: torch.Tensor | QuantizedWeight,
    epilogue: int = EPI_BF16,
    residual: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    mode: int = MODE_AUTO,
    splits: int = 0,
    trace: torch.Tensor | None = None,
    segments: list | None = None,
    cta_trace: torch.Tensor | None = None,
    reduction: int = 0,
    debug: int = 0,
) -> torch.Tensor:
    """``epilogue(a @ w.T)`` on the tcgen05 GEMM: a [M, K] BF16, w [N, K] BF16.

    EPI_BF16 returns BF16 [M, N] (plus ``residual`` before the one rounding), EPI_F32 FP32 [M, N],
    EPI_SWIGLU BF16 [M, N/2] for gate/up weights interleaved in 128-row blocks. A
    ``QuantizedWeight`` runs in its format's contract: ``fp8_block`` and ``nvfp4_a4`` quantize the
    inputs and use the FP8 / block-scaled FP4 tensor cores (W8A8, W4A4); ``fp8_block_w8a16`` and
    ``nvfp4`` dequantize the weights to BF16 tile by tile inside the kernel (W8A16, W4A16).
    ``segments`` [(a1 [M, k1], w1 [N, k1]), ...] (at most two, k a multiple of 64) add
    ``a1 @ w1.T`` and so on into the same FP32 sums before the epilogue (LoRA updates).
    ``trace`` (int64 [8]) and ``cta_trace`` (int64 [4 x CTAs]) receive global-timer milestones.
    ``reduction`` (measurements) makes split-K partials meet in global scratch (1) or the cluster (2);
    ``debug`` (measurements) leaves out the output stores (1) and the accumulator reads (2).
    """
    _rowmajor(a, "a")
    M, K = a.shape
    quant = isinstance(w, QuantizedWeight)
    a_ptr, lda = a.data_ptr(), a.stride(0)
    if quant:
        _rowmajor(w.codes, "codes")
        N = w.rows
        if w.cols != K:
            raise ValueError("inner dimensions differ")
        w_ptr, ldw = w.codes.data_ptr(), w.codes.stride(0) * (1 if w.format.startswith("fp8") else 2)
        qargs = dict(w_format=w.code, w_scale=w.scales.data_ptr(), w_scale_ld=w.scales.stride(0),
                     w_tensor_scale=float(w.tensor_scale), w_scale_rows=1 if w.format == "fp8_rows" else 128)
        if w.format == "nvfp4_a4":
            codes, atoms = quantize_nvfp4_input(a, w.input_scale)
            keep = (codes, atoms)  # noqa: F841 (alive until the launch is enqueued)
            a_ptr, lda = codes.data_ptr(), K
            qargs.update(a_scale=atoms.data_ptr(), w_tensor_scale=_f32(_f32(w.input_scale) * _f32(w.tensor_scale)))
        elif w.format == "fp8_block":
            codes, ascales = quantize_fp8_input(a)
            keep = (codes, ascales)  # noqa: F841
            a_ptr, lda = codes.data_ptr(), K
            padded = w.fp8_gemm_scales()
            qargs.update(a_scale=ascales.data_ptr(), a_scale_ld=ascales.stride(0),
                         w_scale=padded.data_ptr(), w_scale_ld=padded.shape[1])
    else:
        _rowmajor(w, "w")
        if w.dtype != torch.bfloat16:
            raise ValueError("gemm takes BF16 operands")
        N = w.shape[0]
        if w.shape[1] != K:
            raise ValueError("inner dimensions differ")
        w_ptr, ldw = w.data_ptr(), w.stride(0)
        qargs = {}
    if a.dtype != torch.bfloat16:
        raise ValueError("gemm takes BF16 activations")
    cols = N // 2 if epilogue == EPI_SWIGLU else N
    if out is None:
        dtype = torch.float32 if epilogue == EPI_F32 else torch.bfloat16
        out = torch.empty(M, cols, dtype=dtype, device=a.device)
    if residual is not None:
        _rowmajor(residual, "residual")
    s = scratch(a.device)
    native().ops.gemm(
        a_ptr, lda, w_ptr, ldw, M, N, K,
        out.data_ptr(), out.stride(0), _ptr(residual), 0 if residual is None else residual.stride(0),
        epilogue, mode, splits, s.workspace.data_ptr(), s.workspace.numel() * 4,
        s.counters.data_ptr(), s.counters.numel(), s.status.data_ptr(), _stream(),
        0 if trace is None else trace.data_ptr(), **qargs,
        segments=[(sa.data_ptr(), sa.stride(0), sw.data_ptr(), sw.stride(0), sa.shape[1]) for sa, sw in (segments or [])],
        cta_trace=0 if cta_trace is None else cta_trace.data_ptr(), reduction=reduction, debug=debug,
    )
    return out


def rmsnorm(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    residual: torch.Tensor | None = None,
    residual_out: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``RMSNorm(x + residual) * weight``; the rounded sum goes to ``residual_out`` when given."""
    _rowmajor(x, "x")
    rows, cols = x.shape
    out = torch.empty_like(x) if out is None else out
    native().ops.rmsnorm(
        x.data_ptr(), x.stride(0), _ptr(residual), 0 if residual is None else residual.stride(0),
        weight.data_ptr(), out.data_ptr(), out.stride(0), _ptr(residual_out),
        0 if residual_out is None else residual_out.stride(0), rows, cols, float(eps), _stream(),
    )
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, row_begin: int = 0, row_end: int | None = None) -> torch.Tensor:
    rows = ids.numel()
    row_end = table.shape[0] + row_begin if row_end is None else row_end
    out = torch.empty(rows, table.shape[1], dtype=table.dtype, device=table.device)
    native().ops.embedding(ids.data_ptr(), table.data_ptr(), table.stride(0), row_begin, row_end,
                           out.data_ptr(), out.stride(0), rows, table.shape[1], _stream())
    return out


def argmax(logits: torch.Tensor, valid: int | None = None, base: int = 0):
    rows, cols = logits.shape
    idx = torch.empty(rows, dtype=torch.int32, device=logits.device)
    val = torch.empty(rows, dtype=torch.float32, device=logits.device)
    native().ops.argmax(logits.data_ptr(), logits.stride(0), rows, cols,
                        cols if valid is None else valid, base, idx.data_ptr(), val.data_ptr(),
                        _stream())
    return idx, val


def qk_norm_rope_cache(qkv, q_heads, kv_heads, head_dim, q_norm, k_norm, eps, positions, inv_freq,
                       attention_factor, cache, slots):
    rows = qkv.shape[0]
    q = torch.empty(rows, q_heads, head_dim, dtype=torch.bfloat16, device=qkv.device)
    native().ops.qk_norm_rope_cache(
        qkv.data_ptr(), qkv.stride(0), rows, q_heads, kv_heads, head_dim, _ptr(q_norm),
        _ptr(k_norm), float(eps), positions.data_ptr(), inv_freq.data_ptr(),
        float(attention_factor), q.data_ptr(), cache.data_ptr(), slots.data_ptr(), _stream(),
        cache_slots=cache.shape[0] * 16, status=scratch(qkv.device).status.data_ptr())
    return q


def _attn_common(segments: torch.Tensor) -> None:
    if segments.dtype != torch.int32 or segments.dim() != 2 or segments.shape[1] != 5:
        raise ValueError("segments are int32 [n, 5]: row_start, len, cached, table_start, nblocks")


def paged_decode(q, cache, table, segments, kv_heads, max_keys, scale=None, keys_per_split=2048, out=None,
                 counters=None, warps=0, stages=0):
    """Flash-decoding of one-row segments over the paged cache. q: [rows, q_heads, d]. With
    `counters` (int32, zero, one per segment and key/value head) the splits merge in the kernel.
    `warps` (2-4) and `stages` (2-3) pick the CTA shape (0: the engine's defaults); measurements
    compare them."""
    _attn_common(segments)
    rows, q_heads, d = q.shape
    out = torch.empty_like(q) if out is None else out
    s = scratch(q.device)
    n = segments.shape[0]
    splits = (max_keys + keys_per_split - 1) // keys_per_split
    need = n * q_heads * splits
    po = torch.empty(need * d if splits > 1 else 1, dtype=torch.float32, device=q.device)
    pl = torch.empty(need if splits > 1 else 1, dtype=torch.float32, device=q.device)
    native().ops.paged_decode(
        q.data_ptr(), out.data_ptr(), cache.data_ptr(), table.data_ptr(), segments.data_ptr(), n,
        q_heads, kv_heads, d, float(scale if scale is not None else d ** -0.5), po.data_ptr(),
        pl.data_ptr(), need, int(max_keys), keys_per_split, s.status.data_ptr(), _stream(),
        0 if counters is None else counters.data_ptr(), warps, stages, cache.shape[0])
    return out


PREFILL_TILE = 128  # (token, head) rows of a prefill query tile


def prefill_work(segments_cpu, group: int) -> torch.Tensor:
    """(segment, query tile) pairs of the prefill kernel, as int32 [n, 2]."""
    work = []
    for i, (_, length, _, _, _) in enumerate(segments_cpu.tolist()):
        for tile in range((length * group + PREFILL_TILE - 1) // PREFILL_TILE):
            work.append((i, tile))
    return torch.tensor(work, dtype=torch.int32).reshape(-1, 2)


def paged_prefill(q, cache, table, segments, kv_heads, work, scale=None, out=None, tensor_cores=True,
                  causal=True):
    """Attention of segments' rows over their history and themselves (128-row query tiles of
    ``prefill_work``): causal, or with ``causal=False`` bidirectional (every row attends every key
    of its segment, as encoders do). ``cache`` is the layer's pages [blocks, 2, kv_heads, 16, d];
    ``tensor_cores=False`` runs the mma.sync kernel."""
    _attn_common(segments)
    rows, q_heads, d = q.shape
    out = torch.empty_like(q) if out is None else out
    s = scratch(q.device)
    native().ops.paged_prefill(
        q.data_ptr(), out.data_ptr(), cache.data_ptr(), table.data_ptr(), segments.data_ptr(),
        segments.shape[0], q_heads, kv_heads, d, float(scale if scale is not None else d ** -0.5),
        work.data_ptr(), work.shape[0], s.status.data_ptr(), _stream(),
        rows=rows if tensor_cores else 0, cache_blocks=cache.shape[0], bidirectional=not causal)
    return out


# ------------------------------------------------------------------------------ mixture of experts


def moe_route(logits: torch.Tensor, k: int, normalize: bool = True):
    """Top-k routing of BF16 logits [rows, experts]: (ids int32 [rows, k], weights FP32 [rows, k])."""
    _rowmajor(logits, "logits")
    rows, experts = logits.shape
    ids = torch.empty(rows, k, dtype=torch.int32, device=logits.device)
    w = torch.empty(rows, k, dtype=torch.float32, device=logits.device)
    native().ops.moe_route(logits.data_ptr(), logits.stride(0), rows, experts, k, bool(normalize),
                           ids.data_ptr(), w.data_ptr(), _stream())
    return ids, w


def moe_capacity(rows: int, k: int, count: int, tile: int) -> int:
    return (rows * k + count * (tile - 1) + tile - 1) // tile * tile


def moe_align(ids: torch.Tensor, experts: int, tile: int, first: int = 0, count: int | None = None):
    """Groups selections by expert: (pos [rows, k], src [capacity], tile_expert [capacity/tile],
    tiles [1]) for the experts [first, first + count)."""
    rows, k = ids.shape
    count = experts - first if count is None else count
    cap = moe_capacity(rows, k, count, tile)
    dev = ids.device
    pos = torch.empty(rows, k, dtype=torch.int32, device=dev)
    src = torch.empty(cap, dtype=torch.int32, device=dev)
    tile_expert = torch.zeros(cap // tile, dtype=torch.int32, device=dev)
    tiles = torch.zeros(1, dtype=torch.int32, device=dev)
    native().ops.moe_align(ids.data_ptr(), rows, k, experts, first, count, tile, cap, pos.data_ptr(),
                           src.data_ptr(), tile_expert.data_ptr(), tiles.data_ptr(), _stream())
    return pos, src, tile_expert, tiles


def grouped_gemm(a: torch.Tensor, w: torch.Tensor, tiles: torch.Tensor, tile_expert: torch.Tensor, tile: int,
                 epilogue: int = EPI_BF16) -> torch.Tensor:
    """Per-expert ``epilogue(a[rows of e] @ w[e].T)``: a [capacity, K] BF16 sorted by expert (each
    expert's rows padded to ``tile``), w [E, N, K] BF16; rows past the tiles in use are not written."""
    _rowmajor(a, "a")
    E, N, K = w.shape
    M = a.shape[0]
    cols = N // 2 if epilogue == EPI_SWIGLU else N
    out = torch.zeros(M, cols, dtype=torch.float32 if epilogue == EPI_F32 else torch.bfloat16, device=a.device)
    s = scratch(a.device)
    native().ops.gemm(
        a.data_ptr(), a.stride(0), w.data_ptr(), K, M, N, K, out.data_ptr(), out.stride(0), 0, 0,
        epilogue, MODE_SWAP, 1, s.workspace.data_ptr(), s.workspace.numel() * 4, s.counters.data_ptr(),
        s.counters.numel(), s.status.data_ptr(), _stream(), 0,
        group_tiles=tiles.data_ptr(), tile_group=tile_expert.data_ptr(), group_tile=tile, groups=E,
    )
    return out


def moe_gather(x: torch.Tensor, src: torch.Tensor, tiles: torch.Tensor, tile: int) -> torch.Tensor:
    cap = src.shape[0]
    out = torch.zeros(cap, x.shape[1], dtype=x.dtype, device=x.device)
    native().ops.moe_gather(x.data_ptr(), x.stride(0), src.data_ptr(), tiles.data_ptr(), tile, cap,
                            x.shape[1], out.data_ptr(), _stream())
    return out


def moe_combine(y: torch.Tensor, pos: torch.Tensor, weights: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """residual += bf16(sum_j w_j * y[pos_j]) in choice order (in place); returns residual."""
    rows, k = pos.shape
    native().ops.moe_combine(y.data_ptr(), y.stride(0), pos.data_ptr(), weights.data_ptr(), rows, k,
                             residual.shape[1], residual.data_ptr(), residual.stride(0), _stream())
    return residual
