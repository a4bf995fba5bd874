"""SGLang's memory saver on the engine without a GPU: releasing by tag drops the decoder and the
cache and trims the device; resuming loads from the host copy (weights CPU backup) or the files,
weights before the cache, each tag once."""

from types import SimpleNamespace

import pytest

from furiosa_opt_sglang import residency
from furiosa_opt_sglang.platform import Refused


def served(**kw):
    log = []

    def load(source, device):
        log.append(("load", source))
        return SimpleNamespace(cache="spec", source=source)

    def cache(spec, blocks):
        log.append(("cache", blocks))
        return SimpleNamespace(blocks=blocks)

    device = SimpleNamespace(synchronize=lambda: log.append(("sync",)))
    s = residency.Served("/m", device, 64, load=load, checkpoint=lambda p: f"files of {p}",
                         host_copy=lambda p: f"copy of {p}", cache=cache,
                         trim=lambda d: log.append(("trim",)), **kw)
    return s, log


def test_release_and_resume_with_cpu_backup():
    s, log = served(memory_saver=True, cpu_backup=True)
    assert s.model.source == "copy of /m" and s.kv.blocks == 64
    log.clear()
    s.release()
    assert s.model is None and s.kv is None and s.released == {"weights", "kv_cache"}
    assert log[-1] == ("trim",)
    log.clear()
    s.resume()
    assert log == [("load", "copy of /m"), ("cache", 64)]
    assert s.released == set()


def test_without_backup_resume_reads_the_files_and_tags_go_one_by_one():
    s, log = served(memory_saver=True)
    assert s.model.source == "files of /m"
    s.release(["kv_cache"])
    assert s.model is not None and s.kv is None
    log.clear()
    s.resume(["kv_cache"])
    assert log == [("cache", 64)]
    s.release(["weights", "kv_cache"])
    with pytest.raises(RuntimeError, match="after the weights"):
        s.resume(["kv_cache"])
    log.clear()
    s.resume()
    assert log == [("load", "files of /m"), ("cache", 64)]


def test_refusals():
    s, _ = served()
    with pytest.raises(Refused) as e:
        s.release()
    assert e.value.option == "enable_memory_saver"
    s, _ = served(memory_saver=True)
    s.release(["cuda_graph"])  # the engine's graphs go with the weights: nothing of its own
    assert s.released == set()
    with pytest.raises(Refused) as e:
        s.release(["activations"])
    assert e.value.option == "tags"
