"""Sleep mode and weight reloads of the vLLM worker, on stand-ins for the loaded decoder and cache:
what each level keeps, the order tags are released and restored, and the refusals (the
reference's residency: integrations/furiosa-opt-vllm/furiosa_opt_vllm/residency.py)."""

from types import SimpleNamespace

import pytest

from furiosa_opt_vllm import admission, load, residency


class FakeDevice:
    def synchronize(self):
        pass


class FakeModel:
    def __init__(self, source):
        self.source, self.device, self.cache = source, FakeDevice(), "spec"


class FakeCache:
    def __init__(self, spec, blocks):
        self.spec, self.blocks = spec, blocks


@pytest.fixture
def worker(monkeypatch):
    from furiosa_opt_engine import _native
    from furiosa_opt_engine import decoder as dec

    trims = []
    monkeypatch.setattr(_native, "_device_trim", lambda device: trims.append(device))
    monkeypatch.setattr(load, "load_from", lambda ck, device, world, adapters=False, architecture=None: FakeModel(ck))
    monkeypatch.setattr(load, "host_copy", lambda path, config=None: f"copy of {path}")
    monkeypatch.setattr(load, "checkpoint", lambda path, config=None: f"files of {path}")
    monkeypatch.setattr(dec, "Cache", FakeCache)
    w = SimpleNamespace(model_config=SimpleNamespace(enable_sleep_mode=True, model="/m"),
                        parallel_config=SimpleNamespace(tensor_parallel_size=1), engine_device="dev", runner=None,
                        model=FakeModel("copy of /m"), cache=FakeCache("spec", 64), copy="copy of /m", asleep={})
    w.trims = trims
    return w


def test_level_one_keeps_the_copy_and_wakes_from_it(worker):
    residency.sleep(worker, 1)
    assert worker.model is None and worker.cache is None
    assert worker.asleep == {"weights": residency.Weights("copy of /m"), "kv_cache": residency.Storage(64)}
    assert worker.trims == ["dev"]
    residency.wake_up(worker, None)
    assert worker.asleep == {}
    assert worker.model.source == "copy of /m" and worker.cache.blocks == 64


def test_level_two_drops_the_copy_and_reads_the_files(worker):
    residency.sleep(worker, 2)
    assert worker.asleep["weights"] == residency.Weights(None) and worker.copy is None
    residency.wake_up(worker, ["weights"])
    assert "kv_cache" in worker.asleep and worker.model.source == "copy of /m" and worker.copy == "copy of /m"
    residency.wake_up(worker, ["kv_cache"])
    assert worker.asleep == {} and worker.cache.blocks == 64


def test_discard_releases_only_the_named_tag(worker):
    residency.release(worker, ("kv_cache",))
    assert list(worker.asleep) == ["kv_cache"] and worker.model is not None


def test_reload_reads_the_files_again(worker):
    before = worker.model
    residency.reload(worker)
    assert worker.model is not before and worker.model.source == "copy of /m"
    residency.sleep(worker, 1)
    with pytest.raises(RuntimeError, match="requires awake weights"):
        residency.reload(worker)


def test_refusals(worker):
    worker.model_config.enable_sleep_mode = False
    with pytest.raises(admission.Refused, match="enable_sleep_mode"):
        residency.sleep(worker, 1)
    worker.model_config.enable_sleep_mode = True
    worker.cache = None
    with pytest.raises(RuntimeError, match="initialize_kv_cache must precede sleep mode"):
        residency.sleep(worker, 1)


def test_health_check_raises_on_a_failed_device():
    from types import SimpleNamespace

    w = SimpleNamespace(engine_device=None)
    residency.check_health(w)  # before load: nothing to check
    calls = []
    w.engine_device = SimpleNamespace(synchronize=lambda: calls.append(1))
    residency.check_health(w)
    assert calls == [1]
    # A device that can be checked without waiting is not synchronized.
    w.engine_device = SimpleNamespace(check=lambda: calls.append(2), synchronize=lambda: calls.append(3))
    residency.check_health(w)
    assert calls == [1, 2]

    def failed():
        raise RuntimeError("the device failed earlier: launch failed")

    w.engine_device = SimpleNamespace(synchronize=failed)
    with pytest.raises(RuntimeError, match="failed earlier"):
        residency.check_health(w)
