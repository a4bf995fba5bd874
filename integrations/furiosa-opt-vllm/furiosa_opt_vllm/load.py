"""Loads the engine decoder a vLLM model config names: a Hugging Face checkpoint directory through
`Checkpoint` and `LoadOptions` (strict, unconverted), on this rank's GPU."""

from __future__ import annotations


def checkpoint(model_path: str, config: dict | None = None):
    """The checkpoint's files, read with `config` instead of its config.json when given."""
    import furiosa_opt_engine as engine

    return engine.Checkpoint(model_path, config)


def host_copy(model_path: str, config: dict | None = None):
    """The checkpoint with every tensor copied into host memory (sleep mode's copy)."""
    return checkpoint(model_path, config).read()


def overridden(model_path: str, hf_overrides) -> dict | None:
    """The checkpoint's config.json under vLLM's `hf_overrides` (None without overrides). As
    transformers' `PretrainedConfig.update` does, a key replaces the config's value, except that an
    override of a nested sub-config (a value with its own `model_type`) updates its keys."""
    import json
    import os

    from .admission import Refused

    if not hf_overrides:
        return None
    if not isinstance(hf_overrides, dict):
        raise Refused("hf_overrides", "a mapping of config keys; a function of the config is not served")
    with open(os.path.join(model_path, "config.json")) as f:
        config = json.load(f)
    for key, value in hf_overrides.items():
        old = config.get(key)
        if isinstance(value, dict) and isinstance(old, dict) and "model_type" in old:
            config[key] = {**old, **value}
        else:
            config[key] = value
    return config


def architectures(model_path: str) -> list[str]:
    """The classes the checkpoint's config.json declares."""
    import json
    import os

    with open(os.path.join(model_path, "config.json")) as f:
        return list(json.load(f).get("architectures") or [])


def batch_invariant() -> bool:
    """Whether vLLM runs batch invariant (`VLLM_BATCH_INVARIANT=1`): a request's tokens and rows
    then keep their bits whatever other requests share its steps."""
    import os

    return os.environ.get("VLLM_BATCH_INVARIANT", "0").strip().lower() in ("1", "true")


def load_from(ck, device, world: int, adapters: bool = False, architecture: str | None = None,
              invariant: bool | None = None):
    import furiosa_opt_engine as engine

    opts = engine.LoadOptions()
    if architecture is not None:
        opts = opts.architecture(architecture)
    if world > 1:
        opts = opts.chips(world)
    if adapters:
        opts = opts.adapters()
    if batch_invariant() if invariant is None else invariant:
        opts = opts.batch_invariant()
    return opts.load(ck, device)


def replica_chips(local_rank: int, tp_rank: int, tp: int, dp_rank: int = 0, visible: str | None = None) -> list:
    """GPU ordinals of this worker's replica (`tp` chips, one per worker). FURIOSA_VISIBLE_CHIPS
    (comma-separated ordinals) lists every replica's chips in turn: replica i takes chips
    i*tp .. (i+1)*tp (the reference's data parallelism); without it the replica is the `tp`
    consecutive GPUs whose tp_rank-th is this worker's local GPU."""
    if visible:
        chips = [int(c) for c in visible.split(",") if c.strip()]
        mine = chips[dp_rank * tp : (dp_rank + 1) * tp]
        if len(mine) != tp:
            raise ValueError(f"FURIOSA_VISIBLE_CHIPS lists {len(chips)} chips; replica {dp_rank} of "
                             f"{tp} chips needs {(dp_rank + 1) * tp}")
        return mine
    first = local_rank - tp_rank
    if first < 0:
        raise ValueError(f"local rank {local_rank} cannot hold tensor-parallel rank {tp_rank}")
    return list(range(first, first + tp))


def load(model_path: str, rank: int, world: int, keep_copy: bool = False, chips: list | None = None,
         group=None, adapters: bool = False, architecture: str | None = None, config: dict | None = None):
    """(decoder, device, host copy or None): this worker's chip of its replica (`chips`, its
    tensor-parallel `rank` of `world`, joined in `group`); a load under sleep mode keeps the host
    copy it loaded. `architecture` overrides the config's class (a causal checkpoint pooled as its
    base model); `config` replaces the checkpoint's config.json (vLLM's overrides applied)."""
    import furiosa_opt_engine as engine

    chips = chips if chips is not None else list(range(world))
    device = engine.Device(engine.Placement(chips, range(8)), rank=rank if world > 1 else 0)
    if world > 1:
        from furiosa_opt_models_b200.parallel import tp

        tp.set_group(group)
    ck = host_copy(model_path, config) if keep_copy else checkpoint(model_path, config)
    return load_from(ck, device, world, adapters, architecture), device, (ck if keep_copy else None)
