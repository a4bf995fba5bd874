"""KV-cache offloading to host memory for vLLM, over the engine's own cache.

vLLM's offloading connector keeps its scheduler side (which blocks are stored on the host, LRU
eviction, when a request waits for its blocks to come back) and calls worker-side handlers to move
blocks. The engine owns the cache storage (`decoder.Cache`, one device buffer a layer, a block one
page of `Pool.bytes`), so the handlers here copy whole pages between those buffers and one pinned
host pool with the engine's own `Transfer`s, on the engine's stream: a store issued after a call
follows the call's kernels, a load issued before a call precedes them.

Failures follow the reference plugin's offload contract (its offload/worker.py and the serving
documentation's failure notes): a copy that fails poisons the offloaded memory (every later
transfer reports failure), a failed load fails its requests (`kv_load_failure_policy` must be
"fail"), and `wait` raises a failed copy only after every copy it waits for has ended.

Enable with vLLM's kv_transfer_config:
    {"kv_connector": "FuriosaOffloadingConnector", "kv_connector_module_path": "furiosa_opt_vllm.offload",
     "kv_role": "kv_both", "kv_connector_extra_config": {"cpu_bytes_to_use": <bytes>}}
"""

from __future__ import annotations

import dataclasses
import time

# The engine cache of this worker, set before the connector registers its handlers.
_cache = None

# Blocks this process's handlers copied each way (monitoring and tests).
STATS = {"stored_blocks": 0, "loaded_blocks": 0}


def attach(cache) -> None:
    global _cache
    _cache = cache


class HostPool:
    """Pinned host pages: block b of layer l at (b * layers + l) * page bytes."""

    def __init__(self, engine, blocks: int, layers: int, page: int):
        import numpy as np

        self.blocks, self.layers, self.page = blocks, layers, page
        self.buffer = engine.HostBuffer(np.zeros(max(blocks * layers * page, 1), dtype=np.uint8))
        self.poisoned = False

    def slot(self, block: int, layer: int):
        return self.buffer.slice((block * self.layers + layer) * self.page, self.page)


@dataclasses.dataclass
class Finished:
    """A finished job, with the fields of vLLM's TransferResult (which its offloading worker reads)."""

    job_id: int
    success: bool
    transfer_size: int | None = None
    transfer_time: float | None = None
    transfer_type: tuple[str, str] | None = None


def _result(**kw) -> Finished:
    return Finished(**kw)


class PageCopies:
    """An offloading handler (vLLM's OffloadingHandler interface): copies pages one way between
    the engine cache and the host pool; a job finishes when its last transfer has."""

    def __init__(self, cache, pool: HostPool, to_host: bool):
        self.cache, self.pool, self.to_host = cache, pool, to_host
        self.jobs: dict[int, tuple[list, int, float]] = {}  # job -> (transfers, bytes, start)
        self.failed: set[int] = set()
        self.done: list = []  # results `wait` settled, reported by the next get_finished

    def _copy(self, gpu_block: int, cpu_block: int) -> list:
        out = []
        for layer, buf in enumerate(self.cache.layers):
            page = buf.slice(gpu_block * self.pool.page, self.pool.page)
            host = self.pool.slot(cpu_block, layer)
            out.append(page.to_host(host) if self.to_host else host.to_hbm(page))
        return out

    def transfer_async(self, job_id: int, spec) -> bool:
        src, dst = spec
        gpu = src if self.to_host else dst
        cpu = dst if self.to_host else src
        gpu_ids, cpu_ids = list(gpu.block_ids), list(cpu.block_ids)
        if len(gpu_ids) != len(cpu_ids):
            raise ValueError(f"offload job {job_id}: {len(gpu_ids)} device blocks for {len(cpu_ids)} host blocks")
        transfers = []
        try:
            if self.pool.poisoned:
                raise RuntimeError("the offloaded memory is poisoned by an earlier failed copy")
            for g, c in zip(gpu_ids, cpu_ids):
                transfers += self._copy(int(g), int(c))
            STATS["stored_blocks" if self.to_host else "loaded_blocks"] += len(gpu_ids)
        except Exception:  # noqa: BLE001 - a failed submission fails the job, after its issued copies
            self.pool.poisoned = True
            self.failed.add(job_id)
        self.jobs[job_id] = (transfers, len(gpu_ids) * len(self.cache.layers) * self.pool.page, time.perf_counter())
        return True

    def _settle(self, job_id: int, block: bool):
        transfers, size, start = self.jobs[job_id]
        ok = job_id not in self.failed
        for t in transfers:
            if not block and not t.done():
                return None
        for t in transfers:
            try:
                t.wait()
            except Exception:  # noqa: BLE001 - every copy ends before the failure is reported
                ok = False
        if not ok:
            self.pool.poisoned = True
        del self.jobs[job_id]
        self.failed.discard(job_id)
        return _result(job_id=job_id, success=ok, transfer_size=size, transfer_time=time.perf_counter() - start,
                       transfer_type=("GPU", "CPU") if self.to_host else ("CPU", "GPU"))

    def get_finished(self) -> list:
        out, self.done = self.done, []
        for job_id in list(self.jobs):
            r = self._settle(job_id, block=False)
            if r is not None:
                out.append(r)
        return out

    def wait(self, job_ids: set[int]) -> None:
        failed = []
        for job_id in [j for j in job_ids if j in self.jobs]:
            r = self._settle(job_id, block=True)
            if not r.success:
                failed.append(job_id)
            self.done.append(r)
        if failed:
            raise RuntimeError(f"offload jobs {sorted(failed)} failed; the offloaded memory is poisoned")

    def shutdown(self) -> None:
        for job_id in list(self.jobs):
            self._settle(job_id, block=True)


def _spec_class():
    from vllm.v1.kv_offload.base import GPULoadStoreSpec
    from vllm.v1.kv_offload.cpu.common import CPULoadStoreSpec
    from vllm.v1.kv_offload.cpu.spec import CPUOffloadingSpec

    class EngineOffloadingSpec(CPUOffloadingSpec):
        """vLLM's host offloading (its manager, and the host block count from cpu_bytes_to_use)
        with the engine's page copies as the worker-side handlers."""

        def get_handlers(self, kv_caches):
            import furiosa_opt_engine as engine

            if _cache is None:
                raise RuntimeError("the engine cache is not attached to the offloading connector")
            if self._handlers is None:
                page = int(_cache.spec.pools[0].bytes)
                pool = HostPool(engine, self.num_blocks * self.block_size_factor, len(_cache.layers), page)
                self._handlers = (PageCopies(_cache, pool, True), PageCopies(_cache, pool, False))
            store, load = self._handlers
            yield GPULoadStoreSpec, CPULoadStoreSpec, store
            yield CPULoadStoreSpec, GPULoadStoreSpec, load

    return EngineOffloadingSpec


def _connector_class():
    # vLLM's connector module resolves its CUDA platform on import, so the subclass is made when
    # vLLM asks for it (on a GPU host), not when this module is imported.
    from vllm.distributed.kv_transfer.kv_connector.v1.offloading_connector import OffloadingConnector

    class FuriosaOffloadingConnector(OffloadingConnector):
        """vLLM's offloading connector over the engine's cache: the worker side registers the
        engine page copies (there are no vLLM attention layers to read a cache layout from)."""

        def __init__(self, vllm_config, role, kv_cache_config=None):
            extra = vllm_config.kv_transfer_config.kv_connector_extra_config
            extra.setdefault("spec_name", "EngineOffloadingSpec")
            extra.setdefault("spec_module_path", __name__)
            super().__init__(vllm_config, role, kv_cache_config)

        def register_kv_caches(self, kv_caches) -> None:
            worker = getattr(self, "connector_worker", None)
            if worker is not None:
                worker._register_handlers(None)

    return FuriosaOffloadingConnector


_made: dict = {}


def __getattr__(name: str):
    # vLLM imports the connector and spec by name from this module (kv_connector_module_path,
    # spec_module_path); both subclass vLLM classes that need its CUDA platform.
    makers = {"FuriosaOffloadingConnector": _connector_class, "EngineOffloadingSpec": _spec_class}
    if name in makers:
        if name not in _made:
            _made[name] = makers[name]()
        return _made[name]
    raise AttributeError(name)
