"""A host-memory tier for SGLang's hierarchical cache, holding copies of the engine's KV pages.

SGLang's cache controller backs evicted radix-tree pages up to a host pool and loads them back
layer by layer before a request that hits them runs. The engine owns the device pages (one buffer
a layer, a 16-token page one block of `Pool.bytes`), so the host tier keeps each layer's pages in
one pinned buffer, page after page, and moves them with the engine's own copies:

- SGLang names token slots; a transfer moves whole pages, and pages that follow each other on both
  sides move in one copy (`runs`).
- Copies are ordered on the engine's stream after the calls that wrote the pages and before the
  calls that read them, so a load issued before a call is complete when the call reads it.
- A copy that fails poisons the tier: every later transfer is refused, and the failure is raised
  by `wait` only once every copy in flight has ended (the offload contract of the reference's
  integrations/furiosa-opt-sglang/furiosa_opt_sglang/offload.py and its serving notes).

`HostTier` depends on nothing of SGLang's; `host_pool_class()` adapts it to SGLang's HostKVCache
interface when SGLang is importable.
"""

from __future__ import annotations

from . import paging


def pages(indices, size: int = paging.PAGE) -> list[int]:
    """The pages whose token slots `indices` (a 1-D integer sequence) lists, each page whole and its
    slots in order from the page start."""
    slots = [int(s) for s in (indices.tolist() if hasattr(indices, "tolist") else indices)]
    if hasattr(indices, "dim") and indices.dim() != 1:
        raise ValueError("hierarchical cache transfers name token slots by a 1-D tensor")
    if len(slots) % size:
        raise ValueError("hierarchical cache transfers move whole pages")
    out = []
    for i in range(0, len(slots), size):
        first = slots[i]
        if first % size or slots[i : i + size] != list(range(first, first + size)):
            raise ValueError("a hierarchical cache page is a page's consecutive token slots")
        out.append(first // size)
    return out


def runs(device: list[int], host: list[int]) -> list[tuple[int, int, int]]:
    """(device block, host page, pages) runs: consecutive pairs that both step by one."""
    if len(device) != len(host):
        raise ValueError(f"{len(device)} device pages for {len(host)} host pages")
    out: list[list[int]] = []
    for d, h in zip(device, host):
        if out and d == out[-1][0] + out[-1][2] and h == out[-1][1] + out[-1][2]:
            out[-1][2] += 1
        else:
            out.append([d, h, 1])
    return [tuple(r) for r in out]


class HostTier:
    """`pages` host pages of every layer of an engine cache (`storage`: a decoder.Cache)."""

    def __init__(self, engine, storage, pages: int):
        self.storage, self.pages = storage, pages
        self.page_bytes = int(storage.spec.pools[0].bytes)
        self.buffers = [engine.HostBuffer(max(pages * self.page_bytes, 1)) for _ in storage.layers]
        self.poisoned = False
        self.inflight: list = []

    def _submit(self, copies) -> None:
        if self.poisoned:
            raise RuntimeError("the host tier is poisoned by an earlier failed copy")
        try:
            for make in copies:
                self.inflight.append(make())
        except Exception:
            self.poisoned = True
            raise

    def _check(self, block: int, page: int, n: int) -> None:
        if page < 0 or page + n > self.pages or block < 0 or block + n > int(self.storage.blocks):
            raise ValueError(f"pages {page}..{page + n} / blocks {block}..{block + n} out of range")

    def backup(self, device_indices, host_indices) -> None:
        """Copies the device pages of `device_indices` into the host pages of `host_indices`, every layer."""
        moved = runs(pages(device_indices), pages(host_indices))
        size = self.page_bytes
        copies = []
        for layer, buf in zip(self.storage.layers, self.buffers):
            for block, page, n in moved:
                self._check(block, page, n)
                copies.append(lambda layer=layer, buf=buf, block=block, page=page, n=n:
                              layer.slice(block * size, n * size).to_host(buf.slice(page * size, n * size)))
        self._submit(copies)

    def load(self, host_indices, device_indices, layer: int) -> None:
        """Copies one layer's host pages back into its device pages."""
        moved = runs(pages(device_indices), pages(host_indices))
        size, dev, buf = self.page_bytes, self.storage.layers[layer], self.buffers[layer]
        copies = []
        for block, page, n in moved:
            self._check(block, page, n)
            copies.append(lambda block=block, page=page, n=n:
                          buf.slice(page * size, n * size).to_hbm(dev.slice(block * size, n * size)))
        self._submit(copies)

    def wait(self) -> None:
        """Waits for every copy in flight; a failure poisons the tier and is raised after all ended."""
        failed = None
        pending, self.inflight = self.inflight, []
        for t in pending:
            try:
                t.wait()
            except Exception as e:  # noqa: BLE001 - every copy ends before the failure is raised
                failed = failed or e
        if failed is not None:
            self.poisoned = True
            raise RuntimeError("a hierarchical cache copy failed; the host tier is poisoned") from failed


_made: dict = {}


def host_pool_class():
    """SGLang's HostKVCache over a `HostTier` of the engine's token pool (`pools.token_pool_class`)."""
    if "host" in _made:
        return _made["host"]
    from sglang.srt.mem_cache.pool_host import HostKVCache

    class Host(HostKVCache):
        def __init__(self, device_pool, ratio: float, size_gb: int, page_size: int):
            import furiosa_opt_engine as engine

            paging.check_page_size(page_size)
            self.device_pool = device_pool
            storage = device_pool.storage
            per_token = int(storage.spec.pools[0].bytes) * len(storage.layers) // paging.PAGE
            self._engine, self._storage = engine, storage
            super().__init__(dtype=device_pool.dtype, device_capacity_tokens=device_pool.size, size_per_token=per_token,
                             start_layer=0, end_layer=len(storage.layers) - 1, host_to_device_ratio=ratio,
                             host_size=size_gb, page_size=page_size, layout="page_first", pin_memory=False,
                             device="cpu")
            self.tier = HostTier(engine, storage, self.size // paging.PAGE)

        def get_size_per_token(self):
            storage = self.device_pool.storage
            return int(storage.spec.pools[0].bytes) * len(storage.layers) // paging.PAGE

        def init_kv_buffer(self):
            return None  # the tier's pinned buffers hold the pages

        def backup_from_device_all_layer(self, device_pool, host_indices, device_indices, io_backend):
            self.tier.backup(device_indices, host_indices)

        def load_to_device_per_layer(self, device_pool, host_indices, device_indices, layer_id, io_backend, **kw):
            self.tier.load(host_indices, device_indices, layer_id)

        def get_data_page(self, index, flat=True):
            raise NotImplementedError("the engine's host tier serves no storage backend")

        def get_dummy_flat_data_page(self):
            raise NotImplementedError("the engine's host tier serves no storage backend")

        def set_from_flat_data_page(self, index, data_page):
            raise NotImplementedError("the engine's host tier serves no storage backend")

    _made["host"] = Host
    return Host
