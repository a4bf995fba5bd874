"""Loads the engine decoder a vLLM model config names: a Hugging Face checkpoint directory through
`Checkpoint` and `LoadOptions` (strict, unconverted), on this rank's GPU."""

from __future__ import annotations


def load(model_path: str, rank: int, world: int):
    import furiosa_opt_engine as engine

    device = engine.Device(engine.Placement(list(range(world)), range(8)))
    ck = engine.Checkpoint(model_path)
    opts = engine.LoadOptions()
    if world > 1:
        opts = opts.chips(world)
    model = opts.load(ck, device)
    return model, device
