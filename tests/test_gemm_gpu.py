"""The tcgen05 GEMM against an FP32 PyTorch reference, in both operand mappings, with split-K,
every epilogue and shapes that end inside a tile."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from furiosa_opt_models_b200 import ops

    return ops


def _ref(a, w):
    return a.float() @ w.float().T


def _close(out, ref, tol=2e-2):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max error {err} vs scale {scale}"


@pytest.mark.parametrize(
    "M,N,K,mode",
    [
        (128, 256, 64, 1),
        (300, 512, 320, 1),
        (1024, 1024, 1024, 1),
        (515, 776, 2048, 1),
        (1, 256, 128, 2),
        (7, 768, 2048, 2),
        (64, 2048, 2048, 2),
        (100, 1024, 6144, 2),
        (256, 512, 512, 2),
        (64, 4096, 2048, 0),
    ],
)
def test_gemm_bf16(M, N, K, mode):
    ops = _ops()
    torch.manual_seed(M * 7 + N)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    out = ops.gemm(a, w, mode=mode)
    torch.cuda.synchronize()
    ops.scratch().check()
    _close(out, _ref(a, w))


@pytest.mark.parametrize("M,mode", [(64, 2), (200, 1)])
def test_gemm_f32_and_residual(M, mode):
    ops = _ops()
    N, K = 512, 1024
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    out = ops.gemm(a, w, epilogue=ops.EPI_F32, mode=mode)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32
    _close(out, _ref(a, w), 1e-3)
    res = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    out = ops.gemm(a, w, residual=res, mode=mode)
    torch.cuda.synchronize()
    _close(out, _ref(a, w) + res.float())


@pytest.mark.parametrize("M,mode", [(16, 2), (64, 2), (256, 2), (384, 1)])
def test_gemm_swiglu(M, mode):
    ops = _ops()
    inter, K = 768, 1024
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    gate = torch.randn(inter, K, device="cuda", dtype=torch.bfloat16) * 0.05
    up = torch.randn(inter, K, device="cuda", dtype=torch.bfloat16) * 0.05
    # 128-row blocks alternate gate and up.
    w = torch.stack([gate.view(-1, 128, K), up.view(-1, 128, K)], dim=1).reshape(2 * inter, K)
    out = ops.gemm(a, w, epilogue=ops.EPI_SWIGLU, mode=mode)
    torch.cuda.synchronize()
    g = _ref(a, gate).bfloat16().float()
    u = _ref(a, up).bfloat16().float()
    ref = torch.nn.functional.silu(g).bfloat16().float() * u
    assert out.shape == (M, inter)
    _close(out, ref)


def test_gemm_splitk_deterministic():
    ops = _ops()
    a = torch.randn(64, 6144, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(2048, 6144, device="cuda", dtype=torch.bfloat16) * 0.02
    first = ops.gemm(a, w, mode=ops.MODE_SWAP, splits=12)
    for _ in range(3):
        again = ops.gemm(a, w, mode=ops.MODE_SWAP, splits=12)
        torch.cuda.synchronize()
        assert torch.equal(first, again)
    _close(first, _ref(a, w))


@pytest.mark.parametrize("M,N,K,splits", [(64, 4096, 2048, 4), (16, 2048, 6144, 8), (33, 1024, 640, 3), (128, 512, 2048, 5)])
def test_gemm_cluster_splits(M, N, K, splits):
    """Swap mapping with K split across a thread-block cluster (reduced over DSMEM)."""
    ops = _ops()
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    res = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    out = ops.gemm(a, w, mode=ops.MODE_SWAP, splits=splits, residual=res)
    torch.cuda.synchronize()
    ops.scratch().check()
    _close(out, _ref(a, w) + res.float())
    again = ops.gemm(a, w, mode=ops.MODE_SWAP, splits=splits, residual=res)
    torch.cuda.synchronize()
    assert torch.equal(out, again)


@pytest.mark.parametrize("M,mode,epi", [(16, 2, 0), (64, 2, 1), (200, 1, 0), (48, 2, 2), (300, 1, 2)])
def test_gemm_extra_k_segments(M, mode, epi):
    """Extra K segments (the LoRA form [X | Z1 | Z2] x [W | B1 | B2]^T) in every epilogue."""
    ops = _ops()
    torch.manual_seed(M)
    N, K = 768, 1024
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    z1 = torch.randn(M, 128, device="cuda", dtype=torch.bfloat16)
    b1 = torch.randn(N, 128, device="cuda", dtype=torch.bfloat16) * 0.05
    z2 = torch.randn(M, 64, device="cuda", dtype=torch.bfloat16)
    b2 = torch.randn(N, 64, device="cuda", dtype=torch.bfloat16) * 0.05
    out = ops.gemm(a, w, epilogue=epi, mode=mode, segments=[(z1, b1), (z2, b2)])
    torch.cuda.synchronize()
    full = _ref(a, w) + _ref(z1, b1) + _ref(z2, b2)
    if epi == 2:
        blocks = full.view(M, -1, 2, 128)
        from furiosa_opt_models_b200.models import reference as R

        ref = R.swiglu(blocks[:, :, 0].reshape(M, N // 2), blocks[:, :, 1].reshape(M, N // 2))
    else:
        ref = full
    _close(out, ref, 2e-2 if epi != 1 else 1e-3)


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("N,K", [(512, 2048), (770, 264), (4096, 768)])
def test_small_row_projections_stream_weights(M, N, K):
    """One row runs as a weight stream (gemv.cu), more on the tensor-core GEMM: BF16 with a
    residual, FP32 and SwiGLU outputs against the FP32 reference."""
    if M > 1 and N % 8 != 0:
        pytest.skip("the tensor-core GEMM writes 16-byte output rows (N a multiple of 8)")
    ops = _ops()
    from furiosa_opt_models_b200.models import dense, reference

    torch.manual_seed(M * 7 + N)
    a = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    res = torch.randn(M, N, device="cuda").bfloat16()
    ref = _ref(a, w)
    _close(ops.gemm(a, w, epilogue=ops.EPI_F32), ref, 1e-3)
    _close(ops.gemm(a, w, epilogue=ops.EPI_BF16, residual=res), ref + res.float())
    if N % 256 == 0:
        g, u = dense.split_gate_up(w)  # 128-row blocks alternate gate and up
        want = reference.swiglu(_ref(a, g), _ref(a, u))
        _close(ops.gemm(a, w, epilogue=ops.EPI_SWIGLU), want)


@pytest.mark.parametrize("M,N,K", [(1000, 2048, 512), (777, 1000, 320), (4096, 2048, 1024)])
def test_gemm_rows_tma_store_with_residual(M, N, K):
    """Row counts above 256 on the rows mapping, BF16 output through shared memory and TMA stores
    (partial tiles clipped at the matrix edge), with and without the residual; a second call into
    a larger output leaves the columns past N untouched."""
    ops = _ops()
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    res = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    out = ops.gemm(a, w, splits=1)
    torch.cuda.synchronize()
    _close(out, _ref(a, w))
    out = ops.gemm(a, w, residual=res, splits=1)
    torch.cuda.synchronize()
    _close(out, _ref(a, w) + res.float())
    wide = torch.full((M, N + 64), 7.0, device="cuda", dtype=torch.bfloat16)
    ops.gemm(a, w, residual=res, splits=1, out=wide[:, :N])
    torch.cuda.synchronize()
    assert torch.equal(wide[:, :N], out)
    assert bool((wide[:, N:] == 7.0).all())
