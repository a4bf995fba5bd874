"""Worker of the tensor-parallel numerics test: one rank of a torchrun group. Loads a base-model
checkpoint (final-normed hidden rows out) through the public API onto `world` chips, runs a prompt
call keeping every row and decode calls feeding fixed tokens, and (rank 0) saves the hidden rows."""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def main() -> None:
    import datetime

    import torch
    import torch.distributed as dist

    import furiosa_opt_engine as engine
    from furiosa_opt_engine import decoder as dec

    out_path, ckpt, steps = sys.argv[1], sys.argv[2], int(sys.argv[3])
    invariant = len(sys.argv) > 4 and sys.argv[4] == "invariant"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    device = engine.Device(engine.Placement(list(range(world)), range(8)))
    opts = engine.LoadOptions()
    if world > 1:
        opts = opts.chips(world)
    if invariant:
        opts = opts.batch_invariant()
    model = opts.load(engine.Checkpoint(ckpt), device)
    data = torch.load(os.path.join(ckpt, "workload.pt"))
    prompts, fed = data["prompts"], data["fed"]  # prompts[i]: int32 ids; fed[i]: ids of decode steps
    cache = dec.Cache(model.cache, 256)
    blocks = [list(range(40 * i, 40 * (i + 1))) for i in range(len(prompts))]
    toks = [engine.HostTensor.from_dlpack(p).to_hbm(device) for p in prompts]
    out = model.forward([dec.Request([blocks[i]], 0, toks[i], dec.Keep.ALL) for i in range(len(prompts))], cache)
    rows = [torch.from_numpy(out.to_host().numpy()).float()]
    cached = [len(p) for p in prompts]
    for s in range(steps):
        step = engine.HostTensor.from_dlpack(torch.tensor([f[s] for f in fed], dtype=torch.int32)).to_hbm(device)
        reqs = [dec.Request([blocks[i]], cached[i], step[i : i + 1], dec.Keep.LAST) for i in range(len(prompts))]
        rows.append(torch.from_numpy(model.forward(reqs, cache).to_host().numpy()).float())
        cached = [c + 1 for c in cached]
    device.synchronize()
    if rank == 0:
        torch.save(rows, out_path)
    if world > 1:
        from furiosa_opt_models_b200.parallel import tp

        tp.detach(model)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
