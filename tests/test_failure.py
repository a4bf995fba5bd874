"""Failure detection on the host, as CPU ranks over gloo: a rank that dies before the tensor-parallel
heap exchange ends its peers' exchange with an error (bounded by the process group's timeout)
before any of their kernels could wait on it."""

import datetime
import multiprocessing as mp
import os
import socket

import pytest


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, die: bool, q) -> None:
    import torch.distributed as dist

    from furiosa_opt_models_b200.parallel import tp

    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=5))
    if die and rank == world - 1:
        os._exit(3)  # this rank dies between steps, with nothing of its own in flight
    try:
        q.put((rank, "ok", tp.exchange_handles(b"heap-%d" % rank)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", type(e).__name__))


def _run(world: int, die: bool):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, die, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    expected = world - 1 if die else world
    for _ in range(expected):
        results.append(q.get(timeout=60))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(results)


def test_handles_exchange_in_rank_order():
    results = _run(2, die=False)
    assert [r[1] for r in results] == ["ok", "ok"]
    assert results[0][2] == [b"heap-0", b"heap-1"]


@pytest.mark.parametrize("world", [2, 3])
def test_a_dead_rank_ends_the_exchange_with_an_error(world):
    results = _run(world, die=True)
    assert len(results) == world - 1
    assert all(status == "error" for _, status, _ in results), results
