"""Sleep mode and weight reloads for vLLM on the engine.

Device memory goes back to the driver when its owners are dropped: the loaded decoder (weights)
and the KV cache, after which the engine hands its cached device blocks back (`_device_trim`).
Waking rebuilds them. vLLM's sleep API (`sleep`, `wake_up` with tags, `reload_weights`) is served
as the reference plugin serves it (integrations/furiosa-opt-vllm/furiosa_opt_vllm/residency.py
there), with this engine's objects:

- Only a load made under `enable_sleep_mode` can sleep: such a load keeps the checkpoint's tensors
  in host memory (`Checkpoint.read()`). Sleeping at level 1 keeps that host copy for the wake-up;
  level 2, or `discard`, lets it go, and the wake-up opens the checkpoint files instead.
- The KV cache remembers how many blocks it had, so waking allocates it again in one step. What it
  held is lost, which is fine: vLLM sleeps only with no request in flight.
- Tags wake in a fixed order and each counts as awake as soon as it is restored; after a failure a
  second `wake_up` restores only the tags still asleep. Release runs in the opposite order, the cache
  before the weights.
- `reload` frees the served weights' device memory first, then loads the checkpoint files again;
  when the files cannot be read the served weights stay in place.
"""

from __future__ import annotations

from dataclasses import dataclass

from .admission import Refused

TAGS = ("weights", "kv_cache")


@dataclass
class Weights:
    copy: object  # the host copy waking loads from, or None (read the files again)


@dataclass
class Storage:
    blocks: int


def _require(worker) -> None:
    if not worker.model_config.enable_sleep_mode:
        raise Refused("enable_sleep_mode",
                      "sleeps only with enable_sleep_mode, whose loads keep the weights' copy for level 1")
    if worker.model is None and "weights" not in worker.asleep:
        raise RuntimeError("load_model must precede sleep mode")


def _drop_model(worker) -> None:
    """Releases the served weights (every rank in step: a tensor-parallel heap detaches)."""
    model = worker.model
    if model is None:
        return
    model.device.synchronize()
    if worker.parallel_config.tensor_parallel_size > 1:
        from furiosa_opt_models_b200.parallel import tp

        tp.detach(model)
    worker.model = None
    if worker.runner is not None:
        worker.runner.model = None
    del model


def _trim(worker) -> None:
    from furiosa_opt_engine import _native

    _native._device_trim(worker.engine_device)


def sleep(worker, level: int) -> None:
    """Release the weights and the KV cache; level 1 keeps the weights' host copy."""
    release(worker, TAGS, keep_copy=level == 1)


def release(worker, tags, keep_copy: bool = False) -> None:
    """Release the memory of the awake `tags`; released weights keep the host copy if asked."""
    _require(worker)
    for tag in reversed(TAGS):
        if tag not in tags or tag in worker.asleep:
            continue
        if tag == "kv_cache":
            if worker.cache is None:
                raise RuntimeError("initialize_kv_cache must precede sleep mode")
            worker.asleep[tag] = Storage(worker.cache.blocks)
            worker.cache = None
            if worker.runner is not None:
                worker.runner.cache = None
        else:
            worker.asleep[tag] = Weights(worker.copy if keep_copy else None)
            if not keep_copy:
                worker.copy = None
            _drop_model(worker)
    _trim(worker)


def wake_up(worker, tags) -> None:
    """Restore the memory of `tags`, or of every tag."""
    from furiosa_opt_engine import decoder as dec

    from . import load

    for tag in TAGS:
        if tags is not None and tag not in tags:
            continue
        state = worker.asleep.get(tag)
        if state is None:
            continue
        if isinstance(state, Weights):
            copy = state.copy if state.copy is not None else load.host_copy(worker.model_config.model,
                                                                             getattr(worker, "checkpoint_config", None))
            _load(worker, copy)
            worker.copy = copy
        else:
            worker.cache = dec.Cache(worker.model.cache, state.blocks)
            if worker.runner is not None:
                worker.runner.cache = worker.cache
        del worker.asleep[tag]


def reload(worker) -> None:
    """Load the awake weights again from the checkpoint's files."""
    from . import load

    if "weights" in worker.asleep:
        raise RuntimeError("reload_weights requires awake weights; wake them up first")
    # The files are read before the served weights leave the device.
    config = getattr(worker, "checkpoint_config", None)
    source = load.host_copy(worker.model_config.model, config) if worker.model_config.enable_sleep_mode else \
        load.checkpoint(worker.model_config.model, config)
    _drop_model(worker)
    _trim(worker)
    _load(worker, source)
    if worker.model_config.enable_sleep_mode:
        worker.copy = source


def _load(worker, source) -> None:
    """Serve the weights of `source`; LoRA adapters loaded for the previous weights are read again
    when a request names them (pins do not survive)."""
    from . import load, lora

    lora_config = getattr(worker, "lora_config", None)
    worker.model = load.load_from(source, worker.engine_device, worker.parallel_config.tensor_parallel_size,
                                  adapters=lora_config is not None, architecture=getattr(worker, "architecture", None))
    if lora_config is not None:
        worker.adapters = lora.Adapters(lora_config.max_loras, lora_config.max_cpu_loras, worker.model.adapters)
    if worker.runner is not None:
        worker.runner.model = worker.model
        worker.runner.adapters = getattr(worker, "adapters", None)


def check_health(worker) -> None:
    """Raises when the worker's engine device failed (its poison makes every later call raise);
    a worker that has not opened its device yet is healthy. The check does not wait for the steps
    in flight (`Device.check`): a failure inside them shows at the next check after they end, and
    a bounded device wait that gives up ends its step with an error, which poisons the device."""
    device = getattr(worker, "engine_device", None)
    if device is None:
        return
    (device.check if hasattr(device, "check") else device.synchronize)()
