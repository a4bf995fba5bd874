"""Worker of the row-collective test: one rank of a torchrun group. Attaches a tensor-parallel
decoder, runs the all-gather and the exchange of BF16 rows over its peer heap (between decoder
calls) and writes whether every result matched to `<out>.<rank>`."""

import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def part(rank: int, rows: int, cols: int):
    import torch

    r = torch.arange(rows).view(-1, 1)
    c = torch.arange(cols).view(1, -1)
    return ((rank * 37 + r * 5 + c) % 200).to(torch.bfloat16)  # small integers: exact in BF16


def main() -> None:
    import datetime

    import torch
    import torch.distributed as dist

    import furiosa_opt_engine as engine
    from furiosa_opt_engine import _native
    from furiosa_opt_models_b200 import serving
    from furiosa_opt_models_b200.models import configs
    from furiosa_opt_models_b200.parallel import tp

    out_path = sys.argv[1]
    world, rank, local = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    cfg = configs.get("tiny-qwen3-tp")
    device = engine.Device(engine.Placement(list(range(world)), range(8)))
    model = _native._synthetic_decoder(device, cfg, tp=world, rank=rank, seed=3, std=0.05)
    tp.attach(model, device)
    cache = engine.decoder.Cache(model.cache, 64)
    alloc = serving.BlockAllocator(64)
    prompt = torch.arange(1, 20, dtype=torch.int32)
    seq = serving.Sequence(engine.HostTensor.from_dlpack(prompt).to_hbm(device), len(prompt), alloc.take(8))
    serving.prefill(model, cache, [seq], [0])

    def dev(t):
        return engine.HostTensor.from_dlpack(t).to_hbm(device)

    def host(h):
        return torch.from_numpy(h.to_host().numpy()).float()

    results = {}
    for rows, cols in [(3, 8), (16, 256), (40, 64)]:
        got = host(_native._tp_all_gather(model, dev(part(rank, rows, cols))))
        want = torch.cat([part(r, rows, cols) for r in range(world)]).float()
        results[f"all_gather {rows}x{cols}"] = bool(torch.equal(got, want))
        serving.decode(model, cache, [seq])  # a decoder call between collectives
        xr = rows * world
        got = host(_native._tp_exchange(model, dev(part(rank, xr, cols))))
        want = torch.cat([part(r, xr, cols)[rank * rows:(rank + 1) * rows] for r in range(world)], dim=1).float()
        results[f"exchange {xr}x{cols}"] = bool(torch.equal(got, want))
    device.synchronize()
    with open(f"{out_path}.{rank}", "w") as f:
        json.dump(results, f)
    tp.detach(model)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
