"""Paged decode and prefill attention against the FP32 PyTorch reference."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(lengths, cached, q_heads, kv_heads, d, blocks=512, seed=0):
    torch.manual_seed(seed)
    cache = torch.randn(blocks, 2, kv_heads, 16, d, dtype=torch.bfloat16) * 0.5
    perm = torch.randperm(blocks).tolist()
    table, segs, row = [], [], 0
    for n, c in zip(lengths, cached):
        nb = (c + n + 15) // 16
        start = len(table)
        table += perm[:nb]
        perm = perm[nb:]
        segs.append((row, n, c, start, nb))
        row += n
    q = torch.randn(row, q_heads, d, dtype=torch.bfloat16)
    return q, cache, torch.tensor(table, dtype=torch.int32), torch.tensor(segs, dtype=torch.int32)


@pytest.mark.parametrize("q_heads,kv_heads,d", [(16, 8, 128), (32, 8, 128), (8, 8, 64), (64, 8, 128)])
def test_paged_decode(q_heads, kv_heads, d):
    from furiosa_opt_models_b200 import ops
    from furiosa_opt_models_b200.models import reference

    cached = [0, 5, 15, 16, 100, 511, 512, 1000, 2047, 3000]
    q, cache, table, segs = _setup([1] * len(cached), cached, q_heads, kv_heads, d)
    ref = reference.paged_attention(q, cache, table, segs)
    out = ops.paged_decode(q.cuda(), cache.cuda(), table.cuda(), segs.cuda(), kv_heads,
                           max_keys=max(cached) + 1)
    torch.cuda.synchronize()
    err = (out.float().cpu() - ref).abs().max().item()
    assert err < 2e-2, err


@pytest.mark.parametrize("tensor_cores", [True, False], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("q_heads,kv_heads,d", [(16, 8, 128), (32, 8, 128), (8, 8, 64), (64, 8, 128),
                                                (16, 16, 128), (32, 4, 64)])
def test_paged_prefill(q_heads, kv_heads, d, tensor_cores):
    from furiosa_opt_models_b200 import ops
    from furiosa_opt_models_b200.models import reference

    # Chunks with and without history, lengths around the 128-row and 128-key tile edges.
    lengths = [7, 16, 33, 64, 130, 1, 200, 65]
    cached = [0, 0, 20, 100, 0, 40, 300, 127]
    q, cache, table, segs = _setup(lengths, cached, q_heads, kv_heads, d)
    ref = reference.paged_attention(q, cache, table, segs)
    work = ops.prefill_work(segs, q_heads // kv_heads)
    out = ops.paged_prefill(q.cuda(), cache.cuda(), table.cuda(), segs.cuda(), kv_heads, work.cuda(),
                            tensor_cores=tensor_cores)
    torch.cuda.synchronize()
    err = (out.float().cpu() - ref).abs().max().item()
    assert err < 2e-2, err


def test_paged_prefill_long_prompts():
    """Prompts of 1024 and 2047 tokens (16 and 32 K/V tiles): the running maximum, the lazy
    rescale and the two-stage ring over many tiles, on the tensor cores."""
    from furiosa_opt_models_b200 import ops
    from furiosa_opt_models_b200.models import reference

    q, cache, table, segs = _setup([1024, 2047, 300], [0, 0, 1500], 16, 8, 128, blocks=512, seed=1)
    # Scores large enough that later keys raise the maximum by more than 2^8.
    q = q * 4
    ref = reference.paged_attention(q, cache, table, segs)
    work = ops.prefill_work(segs, 2)
    out = ops.paged_prefill(q.cuda(), cache.cuda(), table.cuda(), segs.cuda(), 8, work.cuda())
    torch.cuda.synchronize()
    err = (out.float().cpu() - ref).abs().max().item()
    assert err < 3e-2, err


def test_paged_decode_history_beyond_max_keys():
    """A segment longer than the launch's max_keys has more splits than the scratch was laid out
    for: its row is zeros and the status word records a bad argument; the other rows are exact."""
    from furiosa_opt_models_b200 import ops
    from furiosa_opt_models_b200.models import reference

    cached = [5, 300, 1500]  # max_keys 1024 below: the last row does not fit
    q, cache, table, segs = _setup([1] * 3, cached, 16, 8, 128)
    ref = reference.paged_attention(q, cache, table, segs)
    s = ops.scratch(torch.device("cuda", 0))
    s.status.zero_()
    for split in (512, 1024):  # two splits a row, and one split, each overflowed by the long row
        out = ops.paged_decode(q.cuda(), cache.cuda(), table.cuda(), segs.cuda(), 8, max_keys=1024,
                               keys_per_split=split)
        torch.cuda.synchronize()
        assert int(s.status[0].item()) == 7  # kBadArgument
        s.status.zero_()
        assert torch.count_nonzero(out[2]).item() == 0
        assert (out[:2].float().cpu() - ref[:2]).abs().max().item() < 2e-2


def test_block_ids_past_the_cache_are_refused_on_the_device():
    """A block ID past the cache reads as zeros and records the bad-index status (8) instead of
    reading outside the cache; the prefill kernels treat it the same way."""
    from furiosa_opt_models_b200 import ops

    cached = [40, 100]
    q, cache, table, segs = _setup([1, 1], cached, 16, 8, 128, blocks=64)
    bad = table.clone()
    bad[int(segs[1, 3]) + 2] = 64 + 1000  # past the 64 blocks
    s = ops.scratch(torch.device("cuda", 0))
    s.status.zero_()
    out = ops.paged_decode(q.cuda(), cache.cuda(), bad.cuda(), segs.cuda(), 8, max_keys=101)
    torch.cuda.synchronize()
    assert int(s.status[0].item()) == 8
    assert torch.isfinite(out.float()).all()
    s.status.zero_()
    lengths, cached = [20, 33], [0, 16]
    q, cache, table, segs = _setup(lengths, cached, 16, 8, 128, blocks=64)
    bad = table.clone()
    bad[-1] = -5
    work = ops.prefill_work(segs, 2)
    for tc in (True, False):
        out = ops.paged_prefill(q.cuda(), cache.cuda(), bad.cuda(), segs.cuda(), 8, work.cuda(), tensor_cores=tc)
        torch.cuda.synchronize()
        assert int(s.status[0].item()) == 8, tc
        assert torch.isfinite(out.float()).all()
        s.status.zero_()


@pytest.mark.parametrize("tensor_cores", [True, False], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("q_heads,kv_heads,d", [(16, 8, 128), (8, 8, 64), (32, 4, 64)])
def test_bidirectional_prefill(q_heads, kv_heads, d, tensor_cores):
    """Dense attention over every visible key of a segment (encoders): each row attends the whole
    history and every row of its own chunk, against the FP32 reference without the causal mask."""
    from furiosa_opt_models_b200 import ops
    from furiosa_opt_models_b200.models import reference

    lengths = [7, 64, 130, 200, 1]
    cached = [0, 16, 0, 33, 90]
    q, cache, table, segs = _setup(lengths, cached, q_heads, kv_heads, d)
    ref = reference.paged_attention(q, cache, table, segs, causal=False)
    work = ops.prefill_work(segs, q_heads // kv_heads)
    out = ops.paged_prefill(q.cuda(), cache.cuda(), table.cuda(), segs.cuda(), kv_heads, work.cuda(),
                            tensor_cores=tensor_cores, causal=False)
    torch.cuda.synchronize()
    err = (out.float().cpu() - ref).abs().max().item()
    assert err < 2e-2, err


def test_decode_splits_merged_in_kernel_match_the_merge_kernel():
    """With merge counters the last split of each (segment, key/value head) merges in the decode
    kernel: the same bits as the separate merge kernel, and the counters end at zero."""
    from furiosa_opt_models_b200 import ops

    cached = [0, 100, 255, 256, 700, 1500, 3000]
    q, cache, table, segs = _setup([1] * len(cached), cached, 16, 8, 128)
    args = (q.cuda(), cache.cuda(), table.cuda(), segs.cuda(), 8)
    separate = ops.paged_decode(*args, max_keys=max(cached) + 1, keys_per_split=256)
    counters = torch.zeros(len(cached) * 8, dtype=torch.int32, device="cuda")
    for _ in range(2):
        fused = ops.paged_decode(*args, max_keys=max(cached) + 1, keys_per_split=256, counters=counters)
        torch.cuda.synchronize()
        assert torch.equal(fused, separate)
        assert torch.count_nonzero(counters).item() == 0
