"""Loads the engine decoder a vLLM model config names: a Hugging Face checkpoint directory through
`Checkpoint` and `LoadOptions` (strict, unconverted), on this rank's GPU."""

from __future__ import annotations


def checkpoint(model_path: str):
    import furiosa_opt_engine as engine

    return engine.Checkpoint(model_path)


def host_copy(model_path: str):
    """The checkpoint with every tensor copied into host memory (sleep mode's copy)."""
    return checkpoint(model_path).read()


def load_from(ck, device, world: int):
    import furiosa_opt_engine as engine

    opts = engine.LoadOptions()
    if world > 1:
        opts = opts.chips(world)
    return opts.load(ck, device)


def load(model_path: str, rank: int, world: int, keep_copy: bool = False):
    """(decoder, device, host copy or None): a load under sleep mode keeps the host copy it loaded."""
    import furiosa_opt_engine as engine

    device = engine.Device(engine.Placement(list(range(world)), range(8)))
    ck = host_copy(model_path) if keep_copy else checkpoint(model_path)
    return load_from(ck, device, world), device, (ck if keep_copy else None)
