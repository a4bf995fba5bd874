"""SGLang's request and token pools over the engine's KV cache.

SGLang's scheduler allocates token slots from a paged allocator and records each request's slots
in its request-to-token table; the engine's cache is paged the same way (a 16-token page is one
engine block, slot // 16 its block ID). So the plugin lends SGLang:

- a request pool whose table lives in host memory (the engine reads block IDs from it on the host
  while planning each call) and whose freed rows drop the tokens a greedy step left on the device;
- a token pool (SGLang's KVCache) that owns the engine cache storage and moves token rows to and
  from host memory (SGLang's host snapshots of a request's cache);
- SGLang's paged allocator with host-side slot indices.

The reference's pools: integrations/furiosa-opt-sglang/furiosa_opt_sglang/paging.py:37-118 and
cache.py:53-180. The sizing (`Sizes`) depends on nothing of SGLang's and is tested on its own.
"""

from __future__ import annotations

import dataclasses

from . import paging


@dataclasses.dataclass(frozen=True)
class Sizes:
    """A runner's pool sizes: engine cache blocks (one of them SGLang's dummy page), the token
    slots SGLang schedules, and the requests it runs at once."""

    blocks: int
    tokens: int
    requests: int

    @classmethod
    def plan(cls, free_bytes: int, capacity_bytes: int, fraction: float, block_bytes: int, rows: int,
             max_tokens: int | None = None, max_requests: int | None = None) -> "Sizes":
        """`free_bytes` of the device now free, of `capacity_bytes`; SGLang's `mem_fraction_static`
        of the capacity is the most the weights and cache take together, so the cache gets what is
        free beyond the other (1 - fraction) share; `block_bytes` is one block of every layer."""
        budget = free_bytes - int(capacity_bytes * (1.0 - fraction))
        blocks = max(0, budget // block_bytes)
        capacity = max(0, blocks - 1) * paging.PAGE
        if capacity == 0:
            raise ValueError("no device memory is left for the KV cache; raise mem_fraction_static")
        if max_tokens is not None and not 0 < max_tokens <= capacity:
            raise ValueError(f"max_total_tokens must be in 1..{capacity}")
        tokens = (max_tokens or capacity) // paging.PAGE * paging.PAGE
        return cls(tokens // paging.PAGE + 1, tokens, max_requests or rows)


def rows_to_host(cache, page_bytes: int, layer: int, slots: list[int]) -> list[bytes]:
    """The cache rows of `slots` in `layer` (each row: the token's keys then values, as one engine
    page keeps them K pages then V pages), read from the engine cache page by page."""
    import furiosa_opt_engine as engine

    out = []
    pages: dict[int, bytes] = {}
    half = page_bytes // 2
    row = half // paging.PAGE
    for s in slots:
        b, o = divmod(int(s), paging.PAGE)
        if b not in pages:
            host = engine.HostBuffer(page_bytes)
            cache.layers[layer].slice(b * page_bytes, page_bytes).to_host(host).wait()
            pages[b] = bytes(memoryview(host))
        p = pages[b]
        out.append(p[o * row : (o + 1) * row] + p[half + o * row : half + (o + 1) * row])
    return out


def pooler_output(rows):
    """SGLang's pooler result of the embedding rows [requests, hidden] (the rows themselves when
    SGLang is absent)."""
    try:
        from sglang.srt.layers.pooler import EmbeddingPoolerOutput
    except ImportError:
        return rows
    return EmbeddingPoolerOutput(embeddings=rows)


_made: dict = {}


def request_pool_class():
    """SGLang's ReqToTokenPool in host memory; freeing rows drops their device tokens."""
    if "requests" in _made:
        return _made["requests"]
    from sglang.srt.mem_cache.memory_pool import ReqToTokenPool

    class Requests(ReqToTokenPool):
        def __init__(self, size: int, context: int, steps):
            super().__init__(size, context, "cpu", enable_memory_saver=False)
            self.steps = steps

        def free_rows(self, indices):
            self.steps.release(indices)
            super().free_rows(indices)

        def clear(self):
            self.steps.selected.clear()
            super().clear()

    _made["requests"] = Requests
    return Requests


def token_pool_class():
    """SGLang's KVCache over the engine cache storage (the engine runs attention on it)."""
    if "tokens" in _made:
        return _made["tokens"]
    from sglang.srt.mem_cache.memory_pool import KVCache

    class Tokens(KVCache):
        def __init__(self, storage, layers: int, size: int, dtype):
            super().__init__(size, paging.PAGE, dtype, layers, "cpu", enable_memory_saver=False,
                             start_layer=0, end_layer=layers - 1)
            self.storage = storage
            self.page_bytes = int(storage.spec.pools[0].bytes)

        def get_key_buffer(self, layer_id):
            raise NotImplementedError("the engine owns the cache; host snapshots use get_cpu_copy")

        def get_value_buffer(self, layer_id):
            raise NotImplementedError("the engine owns the cache; host snapshots use get_cpu_copy")

        def get_kv_buffer(self, layer_id):
            raise NotImplementedError("the engine owns the cache; host snapshots use get_cpu_copy")

        def set_kv_buffer(self, *args, **kwargs):
            raise NotImplementedError("the engine writes the cache inside its calls")

        def get_kv_size_bytes(self):
            total = sum(len(layer) for layer in self.storage.layers)
            return total // 2, total // 2

        def get_cpu_copy(self, indices, *args, **kwargs):
            slots = [int(s) for s in indices.tolist()]
            return [rows_to_host(self.storage, self.page_bytes, layer, slots) for layer in range(self.layer_num)]

    _made["tokens"] = Tokens
    return Tokens


def overridden(model_path: str, overrides) -> dict | None:
    """The checkpoint's config.json under SGLang's `json_model_override_args` (a JSON object; None
    without overrides): each key replaces the config's value."""
    import json
    import os

    if not overrides:
        return None
    extra = json.loads(overrides) if isinstance(overrides, str) else overrides
    if not isinstance(extra, dict):
        raise ValueError("json_model_override_args: a JSON object of config keys")
    if not extra:
        return None
    with open(os.path.join(model_path, "config.json")) as f:
        config = json.load(f)
    config.update(extra)
    return config


def bind(model_runner) -> None:
    """Loads the engine decoder of `model_runner`'s model on its GPU and sets SGLang's pools, sizes
    and the plugin's `engine_runner` on it."""
    import furiosa_opt_engine as engine
    import torch
    from furiosa_opt_engine import decoder as dec
    from sglang.srt.mem_cache.allocator import PagedTokenToKVPoolAllocator

    from . import residency
    from .runner import Runner

    args = model_runner.server_args
    # SGLang places tensor-parallel rank r on GPU base_gpu_id + r * gpu_id_step.
    tp, step = int(getattr(args, "tp_size", 1) or 1), int(getattr(args, "gpu_id_step", 1) or 1)
    base = int(getattr(args, "base_gpu_id", 0) or 0)
    rank = (int(model_runner.gpu_id) - base) // step % tp
    first = int(model_runner.gpu_id) - rank
    device = engine.Device(engine.Placement(list(range(first, first + tp)), range(8)), rank=rank if tp > 1 else 0)
    opts = engine.LoadOptions()
    if getattr(args, "enable_deterministic_inference", False):
        opts = opts.batch_invariant()  # a request's tokens keep their bits whatever shares its steps
    config = overridden(model_runner.model_config.model_path, getattr(args, "json_model_override_args", None))
    if tp > 1:
        from furiosa_opt_models_b200.parallel import tp as tensor_parallel

        tensor_parallel.set_group(None)  # SGLang's default process group holds its TP ranks
        opts = opts.chips(tp)
    plan: list = []
    algorithm = str(getattr(args, "speculative_algorithm", None) or "").upper()
    # A draft model loads first, so that the target's cache is sized from what it leaves free.
    draft = opts.load(engine.Checkpoint(args.speculative_draft_model_path), device) if algorithm == "STANDALONE" else None

    def block_bytes_of(spec) -> int:
        # One block of every layer: each group's layers take a page of their pool's format.
        return sum(int(spec.pools[g.pool].bytes) * len(g.layers) for g in spec.groups)

    def blocks(decoder) -> int:
        # The draft's cache has the target's block count, so a block costs both.
        block_bytes = block_bytes_of(decoder.cache) + (block_bytes_of(draft.cache) if draft is not None else 0)
        plan.append(Sizes.plan(int(device.available), int(device.capacity), float(model_runner.mem_fraction_static),
                               max(block_bytes, 1), int(decoder.rows), getattr(args, "max_total_tokens", None),
                               getattr(args, "max_running_requests", None)))
        return plan[-1].blocks

    served = residency.Served(
        model_runner.model_config.model_path, device, blocks, load=opts.load,
        checkpoint=lambda path: engine.Checkpoint(path, config),
        host_copy=lambda path: engine.Checkpoint(path, config).read(), cache=dec.Cache,
        trim=lambda d: engine._native._device_trim(d),
        memory_saver=bool(getattr(args, "enable_memory_saver", False)),
        cpu_backup=bool(getattr(args, "enable_weights_cpu_backup", False)))
    sizes, storage = plan[-1], served.kv
    model_runner.served = served
    model_runner.engine_runner = Runner(served.model, device, storage)
    if algorithm:
        from . import speculative

        width = speculative.width_of(args)
        proposer = (speculative.ngram_of(args, width) if algorithm == "NGRAM" else
                    speculative.DraftModel(draft, dec.Cache(draft.cache, sizes.blocks), width - 1))
        model_runner.engine_runner.speculation = speculative.Speculation(proposer, width)
    model_runner.max_total_num_tokens = sizes.tokens
    model_runner.max_running_requests = sizes.requests
    model_runner.kv_cache_dtype = torch.bfloat16
    context = int(model_runner.model_config.context_len)
    model_runner.req_to_token_pool = request_pool_class()(sizes.requests, context, model_runner.engine_runner.steps)
    layers = len(storage.layers)
    model_runner.token_to_kv_pool = token_pool_class()(storage, layers, sizes.tokens, torch.bfloat16)
    model_runner.token_to_kv_pool_allocator = PagedTokenToKVPoolAllocator(
        sizes.tokens, paging.PAGE, torch.bfloat16, "cpu", model_runner.token_to_kv_pool, need_sort=False)
