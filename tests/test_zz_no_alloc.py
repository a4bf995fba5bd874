"""The allocation-free decode attention entry point, called through its exported C symbol.

`foa_paged_decode_noalloc` (declared in csrc/kernels/noalloc.h) serves callers that cannot
allocate device memory while they run (fixed memory budgets, foreign memory pools, plain C plug-in
interfaces): its split partials live in a fixed array inside the library. This test checks it
against the regular decode attention entry point on two calls in a row (head sizes 64 and 128,
one split and several), and checks that an oversized call is refused without a launch.
The file sorts last so that a run stopping at the first failure has already run every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, TOO_LARGE = 0, -3


def _entry():
    import furiosa_opt_engine._native as native

    lib = ctypes.CDLL(native.__file__)
    fn = lib.foa_paged_decode_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int]
    return fn


LONG = [0, 5, 511, 512, 700, 1500, 2047, 4000]
SHORT = [0, 5, 100, 300, 511]  # every history fits one 512-key split


def _inputs(q_heads=16, kv_heads=8, d=128, blocks=600, seed=0, cached=LONG):
    torch.manual_seed(seed)
    cache = torch.randn(blocks, 2, kv_heads, 16, d, dtype=torch.bfloat16, device="cuda") * 0.5
    perm = torch.randperm(blocks).tolist()
    table, segs = [], []
    for row, c in enumerate(cached):
        nb = (c + 1 + 15) // 16
        segs.append((row, 1, c, len(table), nb))
        table += perm[:nb]
        perm = perm[nb:]
    q = torch.randn(len(cached), q_heads, d, dtype=torch.bfloat16, device="cuda")
    table = torch.tensor(table, dtype=torch.int32, device="cuda")
    segs = torch.tensor(segs, dtype=torch.int32, device="cuda")
    return q, cache, table, segs, max(cached) + 1


def _call(fn, q, cache, table, segs, kv_heads, max_keys, out, split=512):
    err = ctypes.create_string_buffer(256)
    rc = fn(q.data_ptr(), out.data_ptr(), cache.data_ptr(), table.data_ptr(), segs.data_ptr(),
            segs.shape[0], q.shape[1], kv_heads, q.shape[2], q.shape[2] ** -0.5, max_keys, split,
            torch.cuda.current_stream().cuda_stream, err, len(err))
    return rc, err.value.decode()


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("cached", [LONG, SHORT], ids=["splits", "one-split"])
def test_no_alloc_matches_the_regular_entry_point_twice(d, cached):
    from furiosa_opt_models_b200 import ops

    fn = _entry()
    q, cache, table, segs, max_keys = _inputs(d=d, cached=cached)
    expected = ops.paged_decode(q, cache, table, segs, 8, max_keys=max_keys, keys_per_split=512)
    torch.cuda.synchronize()
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        rc, msg = _call(fn, q, cache, table, segs, 8, max_keys, out)
        assert rc == OK, msg
        torch.cuda.synchronize()
        assert not torch.isnan(out.float()).any()
        assert (out.float() - expected.float()).abs().max().item() < 2e-2


def test_no_alloc_near_the_limit():
    """A call whose partials just fit the array runs; one whose padded log-sum-exp part tips it
    over is refused (the size check counts the 256-byte padding)."""
    from furiosa_opt_models_b200 import ops

    fn = _entry()
    q, cache, table, segs, _ = _inputs(q_heads=16, kv_heads=8, d=128)
    n, heads, d = segs.shape[0], 16, 128
    limit = 16 << 20
    # Largest split count whose (lse padded + outputs) still fit: 8 segments x 16 heads = 128 entries a split.
    splits = 1
    while True:
        e = n * heads * (splits + 1)
        if ((e + 63) // 64 * 64 + e * d) * 4 > limit:
            break
        splits += 1
    out = torch.zeros_like(q)
    # Splits of 64 keys over histories of up to 64 * splits keys.
    rc, msg = _call(fn, q, cache, table, segs, 8, 64 * splits, out, split=64)
    assert rc == OK, msg
    expected = ops.paged_decode(q, cache, table, segs, 8, max_keys=64 * splits, keys_per_split=64)
    torch.cuda.synchronize()
    assert (out.float() - expected.float()).abs().max().item() < 2e-2
    rc, msg = _call(fn, q, cache, table, segs, 8, 64 * (splits + 1), out, split=64)
    assert rc == TOO_LARGE, msg


def test_no_alloc_refuses_calls_beyond_its_scratch():
    fn = _entry()
    q, cache, table, segs, _ = _inputs()
    out = torch.zeros_like(q)
    # 8 segments * 16 heads * 4096 splits * 129 floats exceeds 16 MiB.
    rc, msg = _call(fn, q, cache, table, segs, 8, 4096 * 512, out)
    assert rc == TOO_LARGE
    assert "16 MiB" in msg
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0
