"""What the plugin installs into SGLang at startup, each SGLang function it replaces or precedes
beside the reason (the reference's hook table:
integrations/furiosa-opt-sglang/furiosa_opt_sglang/hooks.py:111-173).

SGLang's plugin entry point calls `register()`, which installs every row of `HOOKS` through
SGLang's hook registry. Without SGLang nothing is installed, and the runner serves SGLang-shaped
batches directly (tests and embedders).
"""

from __future__ import annotations

import dataclasses
from typing import Callable

INSTALLED = False


@dataclasses.dataclass(frozen=True)
class Hook:
    target: str  # the SGLang function or class, by its import path
    kind: str  # the registry's hook type: REPLACE, BEFORE, AFTER or AROUND
    make: Callable[[], object]  # builds the installed function or class (imports SGLang lazily)
    reason: str


def _worker():
    from .worker import worker_class

    return worker_class()


def _collect():
    from .steps import collect

    return collect


def _assign():
    from .paging import assign

    return assign


def _validate():
    from .platform import validate_request

    return validate_request


def _speculative():
    from .speculative import create_worker

    return create_worker


def _released():
    from .residency import released

    return released


def _resumed():
    from .residency import resumed

    return resumed


HOOKS = (
    Hook("sglang.srt.managers.tp_worker.TpModelWorker", "REPLACE", _worker,
         "the engine runs the scheduled batches: its model runner loads the decoder and lends SGLang "
         "pools over the engine cache"),
    Hook("sglang.srt.managers.scheduler.Scheduler.process_batch_result", "BEFORE", _collect,
         "an overlapped greedy step's tokens are read from the device before SGLang processes it"),
    Hook("sglang.srt.speculative.spec_info.SpeculativeAlgorithm.create_worker", "REPLACE", _speculative,
         "SGLang's speculative workers run torch draft models; the engine drafts (n-grams or a draft "
         "model) and verifies"),
    Hook("sglang.srt.mem_cache.allocation.assign_req_to_token_pool_func", "REPLACE", _assign,
         "the request-to-token table lives in host memory; SGLang's own writer is a device kernel"),
    Hook("sglang.srt.managers.tokenizer_manager.TokenizerManager._validate_one_request", "BEFORE", _validate,
         "a request with inputs the plugin does not serve is refused before tokenization"),
    Hook("sglang.srt.managers.scheduler_components.weight_updater.SchedulerWeightUpdaterManager."
         "release_memory_occupation", "AFTER", _released,
         "releasing memory by tag drops the engine's weights and cache storage"),
    Hook("sglang.srt.managers.scheduler_components.weight_updater.SchedulerWeightUpdaterManager."
         "resume_memory_occupation", "AFTER", _resumed,
         "resuming memory by tag loads the weights and allocates the cache again"),
)


def register(registry=None, kinds=None) -> int:
    """Installs `HOOKS` through `registry.register(target, function, kind)` (SGLang's HookRegistry
    and HookType by default); returns how many were installed (0 without SGLang)."""
    global INSTALLED
    if registry is None:
        try:
            from sglang.srt.plugins.hook_registry import HookRegistry, HookType
        except ImportError:
            return 0
        registry, kinds = HookRegistry, HookType
    for h in HOOKS:
        kind = getattr(kinds, h.kind) if kinds is not None else h.kind
        registry.register(h.target, h.make(), kind)
    INSTALLED = True
    return len(HOOKS)
