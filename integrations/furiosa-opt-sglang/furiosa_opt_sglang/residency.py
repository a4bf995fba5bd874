"""SGLang's memory saver on the engine (`release_memory_occupation` / `resume_memory_occupation`
with the tags `weights`, `kv_cache` and `cuda_graph`; the reference's
integrations/furiosa-opt-sglang/furiosa_opt_sglang/residency.py).

Device memory is released by dropping what holds it (the loaded decoder, the KV cache) and
returning the engine's cached device blocks to the driver; resuming loads or allocates it again.

- Releasing needs `--enable-memory-saver`; without it SGLang's own allocator releases nothing
  either, and so neither does the plugin.
- With `--enable-weights-cpu-backup` the load keeps a host copy of the checkpoint's tensors
  (`Checkpoint.read()`) and resuming loads from it; without it resuming reads the files again.
- A released cache keeps its block count and comes back empty (SGLang flushes its radix cache
  before it releases the KV cache).
- Releasing goes cache first, then weights; resuming weights first, then the cache, one tag after
  another, so a retry after a failure resumes only what is still released.
"""

from __future__ import annotations

from .platform import Refused

TAGS = ("weights", "kv_cache")
# SGLang's tag for its own CUDA graphs: the engine's graphs belong to the decoder and go and come
# back with the weights, so the tag is accepted and does nothing of its own.
GRAPHS = "cuda_graph"


class Served:
    """The engine objects one SGLang scheduler serves on its device.

    `load(source, device)` loads a decoder from a checkpoint or its host copy, `checkpoint(path)`
    opens the files and `host_copy(path)` reads them into host memory; `cache(spec, blocks)`
    allocates a KV cache; `trim(device)` returns the engine's cached device blocks to the driver.
    `blocks` is the cache's block count, or a function of the loaded decoder that sizes it.
    """

    def __init__(self, path, device, blocks: int, *, load, checkpoint, host_copy, cache, trim,
                 memory_saver: bool = False, cpu_backup: bool = False):
        self.path, self.device, self.blocks = path, device, blocks
        self._load, self._checkpoint, self._host_copy = load, checkpoint, host_copy
        self._cache, self._trim = cache, trim
        self.memory_saver, self.cpu_backup = memory_saver, cpu_backup
        self.copy = host_copy(path) if cpu_backup else None
        self.model = load(self.copy if self.copy is not None else checkpoint(path), device)
        if callable(blocks):
            self.blocks = blocks(self.model)
        self.kv = cache(self.model.cache, self.blocks)
        self.released: set[str] = set()

    def _tags(self, tags) -> list[str]:
        tags = list(TAGS) if tags is None else list(tags)
        for t in tags:
            if t not in TAGS and t != GRAPHS:
                raise Refused("tags", f"{t}: the memory saver releases {', '.join(TAGS)} (and {GRAPHS})")
        return tags

    def release(self, tags=None) -> None:
        if not self.memory_saver:
            raise Refused("enable_memory_saver", "memory is released only under the memory saver")
        tags = self._tags(tags)
        if "kv_cache" in tags and "kv_cache" not in self.released:
            self.device.synchronize()
            self.kv = None
            self.released.add("kv_cache")
        if "weights" in tags and "weights" not in self.released:
            self.device.synchronize()
            self.model = None
            self.released.add("weights")
        self._trim(self.device)

    def resume(self, tags=None) -> None:
        tags = self._tags(tags)
        if "weights" in tags and "weights" in self.released:
            source = self.copy if self.copy is not None else self._checkpoint(self.path)
            self.model = self._load(source, self.device)
            self.released.discard("weights")
        if "kv_cache" in tags and "kv_cache" in self.released:
            if self.model is None:
                raise RuntimeError("the KV cache resumes after the weights it follows")
            self.kv = self._cache(self.model.cache, self.blocks)
            self.released.discard("kv_cache")


def _rebind(model_runner) -> None:
    """Points the plugin's runner and SGLang's token pool at what the served objects hold now."""
    served = model_runner.served
    model_runner.engine_runner.model = served.model
    model_runner.engine_runner.cache = served.kv
    pool = getattr(model_runner, "token_to_kv_pool", None)
    if pool is not None and hasattr(pool, "storage"):
        pool.storage = served.kv


def released(_result, updater, request) -> None:
    """After SGLang's `release_memory_occupation`: release the request's tags on the engine."""
    model_runner = updater.tp_worker.model_runner
    model_runner.served.release(getattr(request, "tags", None))
    _rebind(model_runner)


def resumed(_result, updater, request) -> None:
    """After SGLang's `resume_memory_occupation`: load or allocate the request's tags again."""
    model_runner = updater.tp_worker.model_runner
    model_runner.served.resume(getattr(request, "tags", None))
    _rebind(model_runner)
