"""Worker of the tensor-parallel parity test: one rank of a torchrun group. Runs the same synthetic
decoder at TP=world and writes the greedy tokens of a prefill and decode steps to a JSON file."""

import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def main() -> None:
    import datetime

    import torch
    import torch.distributed as dist

    import furiosa_opt_engine as engine
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import configs
    from furiosa_opt_models_b200.parallel import tp

    out_path, model_name, steps = sys.argv[1], sys.argv[2], int(sys.argv[3])
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    cfg = configs.get(model_name)
    device = engine.Device(engine.Placement(list(range(world)), range(8)))
    model = engine._native._synthetic_decoder(device, cfg, tp=world, rank=rank, seed=3, std=0.05)
    if world > 1:
        tp.attach(model, device)
    lengths = [7, 16, 33, 300, 64]
    gen = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg["vocab"], (n,), generator=gen, dtype=torch.int32) for n in lengths]
    cache = engine.decoder.Cache(model.cache, 256)
    alloc = serving.BlockAllocator(256)
    seqs = [serving.Sequence(engine.HostTensor.from_dlpack(p).to_hbm(device), len(p), alloc.take(40))
            for p in prompts]
    out = serving.prefill(model, cache, seqs, list(range(len(seqs))))
    tokens = [[t] for t in out.to_host().numpy().tolist()]
    for _ in range(steps):
        out = serving.decode(model, cache, seqs)
        for i, t in enumerate(out.to_host().numpy().tolist()):
            tokens[i].append(t)
    device.synchronize()
    if rank == 0:
        with open(out_path, "w") as f:
            json.dump(tokens, f)
    if world > 1:
        tp.detach(model)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
