"""Worker of tests/test_gpu_distributed_optimizer.py, run under torch.distributed.run
with one rank per GPU: DistributedIFKFAC on batch shards against IFKFAC on the
full batch in one process (on every rank: each owner checks its layers' factors),
and the ranks' parameters against each other.
Prints one JSON line on rank 0."""
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from ifkfac_b200.distributed import DistributedIFKFAC  # noqa: E402
from ifkfac_b200.ifkfac import IFKFAC  # noqa: E402


def make_model(dev):
    torch.manual_seed(0)
    return nn.Sequential(nn.Linear(32, 64), nn.Tanh(), nn.Linear(64, 48), nn.Tanh(), nn.Linear(48, 10)).to(dev)


def main():
    prec = int(sys.argv[1])
    steps = 5
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    g = torch.Generator().manual_seed(1)
    X = torch.randn(512, 32, generator=g).to(dev)
    Y = torch.randint(0, 10, (512,), generator=g).to(dev)
    shard = slice(rank * 512 // world, (rank + 1) * 512 // world)
    kw = dict(lr=5e-2, damping=1e-2, factor_update_freq=2, momentum=0.9, precision=prec)
    model = make_model(dev)
    dopt = DistributedIFKFAC(model, **kw)
    for _ in range(steps):
        dopt.zero_grad()
        F.cross_entropy(model(X[shard]), Y[shard]).backward()
        dopt.step()
    torch.cuda.synchronize()
    flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
    every = [torch.empty_like(flat) for _ in range(world)]
    dist.all_gather(every, flat)
    same = all(torch.equal(every[0], e) for e in every)
    # the single-process reference on every rank; each rank checks the factors of its own layers
    ref = make_model(dev)
    opt = IFKFAC(ref, **kw)
    for _ in range(steps):
        opt.zero_grad()
        F.cross_entropy(ref(X), Y).backward()
        opt.step()
    torch.cuda.synchronize()
    mine = [(m, r) for m, r in zip(dopt.hooks.linear_layers, opt.hooks.linear_layers) if dopt.owner[m] == rank]
    ferr = max([float((dopt._factors[m][i].float() - opt._factors[r][i].float()).norm()
                      / opt._factors[r][i].float().norm()) for m, r in mine for i in (0, 1)] + [0.0])
    held = sorted(m_i for m_i, m in enumerate(dopt.hooks.linear_layers) if m in dopt._factors)
    owned = sorted(m_i for m_i, m in enumerate(dopt.hooks.linear_layers) if dopt.owner[m] == rank)
    t = torch.tensor([ferr, float(held != owned)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        werr = max(float((a - b).norm() / b.norm()) for a, b in zip(model.parameters(), ref.parameters()))
        owners = sorted(set(dopt.owner.values()))
        print(json.dumps({"same_on_ranks": same, "weight_rel_err": werr, "factor_rel_err": float(t[0]),
                          "factors_on_owners_only": float(t[1]) == 0.0, "owners": owners, "world": world}),
              flush=True)
    opt.cleanup()
    dopt.cleanup()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
