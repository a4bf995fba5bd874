"""Failure detection on one GPU without a GPU fault: a bounded device wait that runs out (a flag
nothing sets) records its status and returns, the context still usable; host-injected launch and
copy failures poison the device as the real ones would, and a fresh device opens afterwards."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports():
    from furiosa_opt_engine import _native

    flag = torch.zeros(1, dtype=torch.int64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    _native.ops.wait_probe(flag.data_ptr(), 1, 50_000_000, status.data_ptr(), stream)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 >= 0.05
    assert status.item() == 5  # the peer-timeout code
    # The flag raised: the wait returns at once and records nothing.
    status.zero_()
    flag.fill_(1)
    _native.ops.wait_probe(flag.data_ptr(), 1, 50_000_000, status.data_ptr(), stream)
    torch.cuda.synchronize()
    assert status.item() == 0


def _decoder():
    import furiosa_opt_engine as engine
    from furiosa_opt_engine import _native
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import configs

    cfg = configs.get("tiny-qwen3")
    device = engine.Device(engine.Placement([0], range(8)))
    model = _native._synthetic_decoder(device, cfg, seed=0, std=0.02)
    cache = engine.decoder.Cache(model.cache, 16)
    alloc = serving.BlockAllocator(16)
    prompt = torch.randint(0, cfg["vocab"], (9,), dtype=torch.int32)
    seq = serving.Sequence(engine.HostTensor.from_dlpack(prompt).to_hbm(device), 9, alloc.take(4))
    return engine, device, model, cache, seq


def test_a_peer_timeout_status_raises_when_results_are_read():
    from furiosa_opt_engine import _native
    from furiosa_opt_models_b200 import serving

    engine, device, model, cache, seq = _decoder()
    out = serving.prefill(model, cache, [seq], [0])
    status, stream = _native._device_status(device)
    flag = torch.zeros(1, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()  # the flag is zero before the engine's stream waits on it
    _native.ops.wait_probe(flag.data_ptr(), 1, 10_000_000, status, stream)
    with pytest.raises(RuntimeError, match="a peer rank never raised its flag"):
        out.to_host()
    with pytest.raises(RuntimeError, match="the device failed earlier"):
        serving.decode(model, cache, [seq])


def test_injected_launch_failure_poisons_the_device():
    from furiosa_opt_engine import _native
    from furiosa_opt_models_b200 import serving

    engine, device, model, cache, seq = _decoder()
    _native._fault_inject(device, "launch", 5)
    with pytest.raises(RuntimeError, match="launch rejected"):
        serving.prefill(model, cache, [seq], [0])
    with pytest.raises(RuntimeError, match="the device failed earlier"):
        serving.prefill(model, cache, [seq], [0])
    # The drill made no GPU fault: a new device on the same GPU serves.
    engine2, device2, model2, cache2, seq2 = _decoder()
    assert serving.prefill(model2, cache2, [seq2], [0]).to_host().numpy().shape == (1,)


def test_injected_copy_failure_poisons_the_device():
    import furiosa_opt_engine as engine
    from furiosa_opt_engine import _native

    device = engine.Device(engine.Placement([0], range(8)))
    _native._fault_inject(device, "copy", 0)
    with pytest.raises(RuntimeError, match="injected fault"):
        engine.HostTensor.from_dlpack(torch.arange(8, dtype=torch.int32)).to_hbm(device)
    with pytest.raises(RuntimeError, match="the device failed earlier"):
        engine.HostTensor.from_dlpack(torch.arange(8, dtype=torch.int32)).to_hbm(device)
