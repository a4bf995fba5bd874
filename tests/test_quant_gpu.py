"""Quantized weights on the device: the FP8 block and NVFP4 quantizers bit for bit against the
PyTorch restatement, and the tcgen05 GEMM with on-the-fly dequantization (W8A16 / W4A16) against
an FP32 product with the dequantized weights."""

import dataclasses

import pytest
import torch

from furiosa_opt_models_b200.models import reference as R

pytestmark = pytest.mark.gpu


def _ops():
    from furiosa_opt_models_b200 import ops

    return ops


def _close(out, ref, tol=2e-2):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max error {err} vs scale {scale}"


@pytest.mark.parametrize("rows,cols", [(128, 128), (300, 520), (1024, 2048)])
def test_fp8_block_quantizer_bitwise(rows, cols):
    ops = _ops()
    torch.manual_seed(rows + cols)
    w = torch.randn(rows, cols, device="cuda", dtype=torch.bfloat16) * 0.03
    w[:128, :128] = 0  # an all-zero block keeps its floor scale
    q = ops.quantize_fp8_block(w)
    torch.cuda.synchronize()
    codes, scales = R.fp8_block_quantize(w)
    assert torch.equal(q.scales, scales)
    assert torch.equal(q.codes, codes)


@pytest.mark.parametrize("rows,cols", [(64, 64), (257, 1024), (2048, 4096)])
def test_nvfp4_quantizer_bitwise(rows, cols):
    ops = _ops()
    torch.manual_seed(rows * 3 + cols)
    w = torch.randn(rows, cols, device="cuda", dtype=torch.bfloat16) * 0.02
    q = ops.quantize_nvfp4(w)
    torch.cuda.synchronize()
    packed, s8, ts = R.nvfp4_quantize(w)
    assert q.tensor_scale == pytest.approx(ts, rel=0, abs=0)
    assert torch.equal(q.scales, s8)
    assert torch.equal(q.codes, packed)


def _weights(fmt, N, K, seed):
    ops = _ops()
    torch.manual_seed(seed)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    if fmt == "fp8_block_w8a16":
        q = dataclasses.replace(ops.quantize_fp8_block(w), format=fmt)
        deq = R.fp8_block_dequantize(q.codes, q.scales)
        factor = 1.0
    else:
        q = ops.quantize_nvfp4(w)
        deq = R.nvfp4_dequantize(q.codes, q.scales)
        factor = q.tensor_scale
    return q, deq, factor


@pytest.mark.parametrize("fmt", ["fp8_block_w8a16", "nvfp4"])
@pytest.mark.parametrize(
    "M,N,K,mode,splits",
    [
        (1, 256, 1024, 2, 0),
        (7, 768, 2048, 2, 0),
        (64, 2048, 4096, 2, 0),
        (64, 640, 1024, 2, 1),
        (200, 1024, 2048, 2, 0),
        (300, 512, 1024, 1, 0),
        (1024, 1536, 2048, 1, 0),
    ],
)
def test_quantized_gemm(fmt, M, N, K, mode, splits):
    ops = _ops()
    q, deq, factor = _weights(fmt, N, K, M + N)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    out = ops.gemm(a, q, mode=mode, splits=splits)
    torch.cuda.synchronize()
    ops.scratch().check()
    _close(out, (a.float() @ deq.T) * factor)


@pytest.mark.parametrize("fmt", ["fp8_block_w8a16", "nvfp4"])
@pytest.mark.parametrize("M,mode", [(16, 2), (128, 2), (384, 1)])
def test_quantized_swiglu(fmt, M, mode):
    ops = _ops()
    inter, K = 768, 1024
    q, deq, factor = _weights(fmt, 2 * inter, K, M)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    out = ops.gemm(a, q, epilogue=ops.EPI_SWIGLU, mode=mode)
    torch.cuda.synchronize()
    full = (a.float() @ deq.T) * factor
    blocks = full.view(M, -1, 2, 128)
    ref = R.swiglu(blocks[:, :, 0].reshape(M, inter), blocks[:, :, 1].reshape(M, inter))
    _close(out, ref)


def test_quantized_gemm_f32_epilogue():
    ops = _ops()
    q, deq, factor = _weights("nvfp4", 512, 2048, 5)
    a = torch.randn(32, 2048, device="cuda", dtype=torch.bfloat16)
    out = ops.gemm(a, q, epilogue=ops.EPI_F32)
    torch.cuda.synchronize()
    _close(out, (a.float() @ deq.T) * factor, 1e-3)


# ------------------------------------------------------------------ W4A4 on the block-scaled MMA


@pytest.mark.parametrize("rows,K", [(1, 256), (77, 512), (300, 1024)])
def test_nvfp4_input_quantizer_bitwise(rows, K):
    ops = _ops()
    torch.manual_seed(rows + K)
    x = torch.randn(rows, K, device="cuda", dtype=torch.bfloat16)
    input_scale = float(x.float().abs().max()) / (6 * 448) * 1.3
    codes, atoms = ops.quantize_nvfp4_input(x, input_scale)
    torch.cuda.synchronize()
    ref_codes, ref_s8 = R.nvfp4_quantize_input(x, input_scale)
    assert torch.equal(codes, ref_codes)
    assert torch.equal(atoms, R.nvfp4_scale_atoms(ref_s8))


def test_nvfp4_scale_atoms():
    ops = _ops()
    q = ops.quantize_nvfp4(torch.randn(200, 512, device="cuda", dtype=torch.bfloat16))
    w4 = ops.nvfp4_w4a4(q, 0.01)
    torch.cuda.synchronize()
    assert torch.equal(w4.scales, R.nvfp4_scale_atoms(q.scales))


@pytest.mark.parametrize(
    "M,N,K,mode,epi",
    [
        (1, 256, 1024, 2, 0),
        (48, 512, 2048, 2, 0),
        (100, 768, 1024, 2, 0),
        (200, 1024, 2048, 2, 0),
        (64, 4096, 4096, 2, 1),
        (512, 768, 1024, 1, 0),
        (1024, 2048, 4096, 1, 0),
        (32, 1536, 1024, 2, 2),
        (160, 1536, 1024, 2, 2),
        (384, 1536, 1024, 1, 2),
    ],
)
def test_nvfp4_w4a4_gemm(M, N, K, mode, epi):
    ops = _ops()
    torch.manual_seed(M + N + K)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    input_scale = float(a.float().abs().max()) / (6 * 448)
    q = ops.quantize_nvfp4(w)
    w4 = ops.nvfp4_w4a4(q, input_scale)
    out = ops.gemm(a, w4, epilogue=epi, mode=mode)
    torch.cuda.synchronize()
    ops.scratch().check()
    ac, as8 = R.nvfp4_quantize_input(a, input_scale)
    a_deq = R.nvfp4_dequantize(ac, as8)
    w_deq = R.nvfp4_dequantize(q.codes, q.scales)
    alpha = float(torch.tensor(w4.input_scale, dtype=torch.float32) * torch.tensor(q.tensor_scale, dtype=torch.float32))
    full = (a_deq @ w_deq.T) * alpha
    if epi == 2:
        blocks = full.view(M, -1, 2, 128)
        inter = N // 2
        ref = R.swiglu(blocks[:, :, 0].reshape(M, inter), blocks[:, :, 1].reshape(M, inter))
    else:
        ref = full
    _close(out, ref, 1e-2 if epi != 1 else 1e-4)


# ------------------------------------------------------------------ W8A8 on the FP8 tensor cores


@pytest.mark.parametrize("rows,K", [(1, 128), (77, 512), (300, 2048)])
def test_fp8_input_quantizer_bitwise(rows, K):
    ops = _ops()
    torch.manual_seed(rows + K)
    x = torch.randn(rows, K, device="cuda", dtype=torch.bfloat16)
    x[0, :128] = 0  # an all-zero group keeps its floor scale
    codes, scales = ops.quantize_fp8_input(x)
    torch.cuda.synchronize()
    ref_codes, ref_scales = R.fp8_quantize_input(x)
    assert torch.equal(codes, ref_codes)
    assert torch.equal(scales[:, :rows], ref_scales.T)


@pytest.mark.parametrize(
    "M,N,K,mode,epi,splits",
    [
        (1, 256, 1024, 2, 0, 0),
        (16, 512, 2048, 2, 0, 0),
        (48, 768, 1024, 2, 0, 1),
        (100, 1024, 2048, 2, 0, 0),
        (64, 4096, 4096, 2, 1, 0),
        (200, 640, 1024, 2, 0, 0),
        (512, 768, 1024, 1, 0, 0),
        (1000, 2048, 4096, 1, 0, 0),
        (32, 1536, 1024, 2, 2, 0),
        (100, 1536, 2048, 2, 2, 0),
        (700, 1536, 1024, 0, 2, 0),
    ],
)
def test_fp8_w8a8_gemm(M, N, K, mode, epi, splits):
    ops = _ops()
    torch.manual_seed(M + N + K)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    q = ops.quantize_fp8_block(w)
    out = ops.gemm(a, q, epilogue=epi, mode=mode, splits=splits)
    torch.cuda.synchronize()
    ops.scratch().check()
    full = R.fp8_block_w8a8(a, q.codes, q.scales)
    if epi == 2:
        blocks = full.view(M, -1, 2, 128)
        inter = N // 2
        ref = R.swiglu(blocks[:, :, 0].reshape(M, inter), blocks[:, :, 1].reshape(M, inter))
    else:
        ref = full
    _close(out, ref, 1e-2 if epi != 1 else 1e-4)


# ------------------------------------------------------------------ FP8 quantized at load (W8A16)


@pytest.mark.parametrize("tensor_amax", [None, 0.4])
def test_fp8_rows_quantizer_and_gemm(tensor_amax):
    ops = _ops()
    torch.manual_seed(12)
    w = torch.randn(640, 1024, device="cuda", dtype=torch.bfloat16) * 0.05
    w[3] = 0  # a zero row keeps zero codes
    q = ops.quantize_fp8_rows(w, tensor_amax)
    torch.cuda.synchronize()
    codes, scales = R.fp8_rows_quantize(w, tensor_amax)
    assert torch.equal(q.codes, codes) and torch.equal(q.scales, scales)
    a = torch.randn(48, 1024, device="cuda", dtype=torch.bfloat16)
    for mode in (1, 2):
        out = ops.gemm(a, q, mode=mode)
        torch.cuda.synchronize()
        _close(out, R.quantized_linear(a.float(), q))
