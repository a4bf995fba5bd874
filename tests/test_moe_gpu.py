"""Mixture-of-experts kernels against the PyTorch restatement: routing (ties included), grouping
by expert, the grouped expert GEMMs and the whole block with its choice-order combine."""

import pytest
import torch

from furiosa_opt_models_b200.models import reference as R

pytestmark = pytest.mark.gpu


def _ops():
    from furiosa_opt_models_b200 import ops

    return ops


@pytest.mark.parametrize("rows,experts,k,normalize", [(1, 128, 8, True), (37, 128, 8, False), (300, 64, 4, True),
                                                      (5, 512, 16, True)])
def test_route_matches_reference(rows, experts, k, normalize):
    ops = _ops()
    torch.manual_seed(rows + experts)
    logits = torch.randn(rows, experts, device="cuda").bfloat16()
    # Ties: equal logits (and -0 against +0) go in ascending expert order.
    logits[0, 3] = logits[0, 9] = logits[0].max()
    if rows > 1:
        logits[1, :] = 0.0
        logits[1, 5] = -0.0
    ids, w = ops.moe_route(logits, k, normalize)
    torch.cuda.synchronize()
    rid, rw = R.moe_route(logits, k, normalize)
    assert torch.equal(ids.long(), rid)
    torch.testing.assert_close(w, rw, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("rows,k,experts,first,count,tile", [(64, 8, 128, 0, 128, 16), (300, 8, 128, 32, 16, 64),
                                                             (1000, 4, 64, 0, 64, 128)])
def test_align_groups_stably(rows, k, experts, first, count, tile):
    ops = _ops()
    torch.manual_seed(rows)
    ids = torch.stack([torch.randperm(experts)[:k] for _ in range(rows)]).int().cuda()
    pos, src, tile_expert, tiles = ops.moe_align(ids, experts, tile, first, count)
    torch.cuda.synchronize()
    ids_c, pos_c, src_c = ids.cpu(), pos.cpu(), src.cpu()
    off = 0
    for e in range(count):
        sel = (ids_c == first + e).flatten().nonzero().flatten()  # (row, choice) order
        n = sel.numel()
        for r, flat in enumerate(sel.tolist()):
            assert pos_c.flatten()[flat].item() == off + r
            assert src_c[off + r].item() == flat // k
        assert (src_c[off + n: off + (n + tile - 1) // tile * tile] == -1).all()
        for t in range(off // tile, (off + n + tile - 1) // tile):
            assert tile_expert[t].item() == e
        off += (n + tile - 1) // tile * tile
    assert tiles.item() * tile == off
    nonlocal_ = ((ids_c < first) | (ids_c >= first + count))
    assert (pos_c[nonlocal_] == -1).all()


@pytest.mark.parametrize("T,H,I,E,k,tile", [(16, 256, 256, 8, 2, 16), (200, 512, 768, 16, 4, 64),
                                            (64, 2048, 768, 128, 8, 16)])
def test_moe_block_matches_reference(T, H, I, E, k, tile):
    ops = _ops()
    torch.manual_seed(T + E)
    h = torch.randn(T, H, device="cuda").bfloat16()
    router = (torch.randn(E, H, device="cuda") * 0.05).bfloat16()
    gate_up = (torch.randn(E, 2 * I, H, device="cuda") * 0.05).bfloat16()
    down = (torch.randn(E, H, I, device="cuda") * 0.05).bfloat16()
    residual = torch.randn(T, H, device="cuda").bfloat16()
    logits = ops.gemm(h, router)
    ids, w = ops.moe_route(logits, k, True)
    pos, src, tile_expert, tiles = ops.moe_align(ids, E, tile)
    xs = ops.moe_gather(h, src, tiles, tile)
    act = ops.grouped_gemm(xs, gate_up, tiles, tile_expert, tile, epilogue=ops.EPI_SWIGLU)
    y = ops.grouped_gemm(act, down, tiles, tile_expert, tile)
    out = ops.moe_combine(y, pos, w, residual.clone())
    torch.cuda.synchronize()
    ops.scratch().check()
    ref = R.moe_forward(h, router, gate_up, down, k)
    expect = (residual.float() + ref.float()).bfloat16()
    err = (out.float() - expect.float()).abs().max().item()
    assert err <= 2e-2 * expect.float().abs().max().item(), err


def test_grouped_gemm_per_expert():
    ops = _ops()
    torch.manual_seed(3)
    T, K, N, E, k, tile = 96, 512, 384, 6, 2, 32
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(E, N, K, device="cuda") * 0.05).bfloat16()
    ids = torch.stack([torch.randperm(E)[:k] for _ in range(T)]).int().cuda()
    pos, src, tile_expert, tiles = ops.moe_align(ids, E, tile)
    xs = ops.moe_gather(x, src, tiles, tile)
    y = ops.grouped_gemm(xs, w, tiles, tile_expert, tile, epilogue=ops.EPI_F32)
    torch.cuda.synchronize()
    for t in range(T):
        for j in range(k):
            e = ids[t, j].item()
            ref = x[t].float() @ w[e].float().T
            torch.testing.assert_close(y[pos[t, j].item()], ref, rtol=2e-3, atol=2e-3)
