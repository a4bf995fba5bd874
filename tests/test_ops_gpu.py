"""Memory-bound kernels against FP32 PyTorch references."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from furiosa_opt_models_b200 import ops

    return ops


@pytest.mark.parametrize("rows,cols", [(1, 1024), (37, 2048), (64, 4096), (3, 8192)])
def test_rmsnorm_with_residual(rows, cols):
    ops = _ops()
    x = torch.randn(rows, cols, device="cuda", dtype=torch.bfloat16)
    r = torch.randn(rows, cols, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(cols, device="cuda", dtype=torch.bfloat16)
    res_out = torch.empty_like(x)
    out = ops.rmsnorm(x, w, 1e-6, residual=r, residual_out=res_out)
    torch.cuda.synchronize()
    h = (x.float() + r.float()).bfloat16()
    assert torch.equal(res_out, h)
    hf = h.float()
    ref = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert (out.float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()


def test_embedding_shard():
    ops = _ops()
    table = torch.randn(100, 256, device="cuda", dtype=torch.bfloat16)
    ids = torch.tensor([0, 5, 99, 50, 51], device="cuda", dtype=torch.int32)
    out = ops.embedding(ids, table[50:], row_begin=50, row_end=100)
    torch.cuda.synchronize()
    ref = table[ids.long()].clone()
    ref[:2] = 0
    assert torch.equal(out, ref)


def test_argmax_first_maximum_wins():
    ops = _ops()
    logits = torch.randn(9, 1000, device="cuda")
    logits[0, 10] = 100.0
    logits[0, 500] = 100.0
    logits[1, :] = 0.0
    logits[2, 998:] = 1e9  # padded columns never win
    idx, val = ops.argmax(logits, valid=998)
    torch.cuda.synchronize()
    ref = logits[:, :998].argmax(-1)
    assert idx[0].item() == 10
    assert idx[1].item() == 0
    assert torch.equal(idx.long(), ref)


@pytest.mark.parametrize("head_dim", [64, 128])
def test_qk_norm_rope_cache(head_dim):
    ops = _ops()
    from furiosa_opt_models_b200.models import reference

    rows, qh, kvh = 11, 4, 2
    qkv = torch.randn(rows, (qh + 2 * kvh) * head_dim, device="cuda", dtype=torch.bfloat16)
    qn = torch.randn(head_dim, device="cuda", dtype=torch.bfloat16)
    kn = torch.randn(head_dim, device="cuda", dtype=torch.bfloat16)
    pos = torch.arange(rows, device="cuda", dtype=torch.int32) * 37 + 5
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, head_dim, 2, device="cuda").float() / head_dim))
    blocks = 4
    cache = torch.zeros(blocks, 2, kvh, 16, head_dim, device="cuda", dtype=torch.bfloat16)
    slots = torch.tensor([3, 17, 18, 40, 63, 0, 1, 2, 20, 21, -1], device="cuda", dtype=torch.int32)
    q = ops.qk_norm_rope_cache(qkv, qh, kvh, head_dim, qn, kn, 1e-6, pos, inv_freq, 1.0, cache, slots)
    torch.cuda.synchronize()
    rq, rk, rv = reference.qk_front(qkv.float().cpu(), qh, kvh, head_dim, qn.float().cpu(),
                                    kn.float().cpu(), 1e-6, pos.long().cpu(), inv_freq.cpu())
    assert (q.float().cpu() - rq).abs().max().item() < 5e-2
    c = cache.float().cpu()
    for r, s in enumerate(slots.tolist()):
        if s < 0:
            continue
        b, o = divmod(s, 16)
        assert (c[b, 0, :, o] - rk[r]).abs().max().item() < 5e-2
        assert (c[b, 1, :, o] - rv[r]).abs().max().item() < 2e-2


def test_cache_slots_past_the_cache_write_nothing():
    """A KV write slot at or past blocks * 16 writes nothing and records the bad-index status (8)."""
    ops = _ops()
    from furiosa_opt_models_b200.ops import scratch

    rows, qh, kvh, d = 3, 4, 2, 128
    qkv = torch.randn(rows, (qh + 2 * kvh) * d, device="cuda", dtype=torch.bfloat16)
    pos = torch.arange(rows, device="cuda", dtype=torch.int32)
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, d, 2, device="cuda").float() / d))
    cache = torch.zeros(2, 2, kvh, 16, d, device="cuda", dtype=torch.bfloat16)
    guard = torch.zeros(1 << 16, device="cuda", dtype=torch.bfloat16)  # memory right after, often
    slots = torch.tensor([1, 32, 5000], device="cuda", dtype=torch.int32)
    s = scratch(torch.device("cuda", 0))
    s.status.zero_()
    ops.qk_norm_rope_cache(qkv, qh, kvh, d, None, None, 1e-6, pos, inv_freq, 1.0, cache, slots)
    torch.cuda.synchronize()
    assert int(s.status[0].item()) == 8
    s.status.zero_()
    assert torch.count_nonzero(cache[0, :, :, 1]).item() > 0  # the valid slot was written
    assert torch.count_nonzero(guard).item() == 0
