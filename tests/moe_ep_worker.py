"""Worker for the expert-parallel MoE check (one process per GPU, NCCL).

``python -m torch.distributed.run --nproc-per-node N tests/moe_ep_worker.py
OUT.json``: every rank builds the same seeded experts, keeps its E/N, routes
its own seeded tokens through MoELayerEP; rank 0 runs every rank's tokens
through the single-GPU MoELayer and writes the normwise differences to
OUT.json.  Test infrastructure only.
"""

import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from xanosmerks_b200.moe import MoELayer, MoELayerEP  # noqa: E402
from xanosmerks_b200.ops import GGUFTensor  # noqa: E402
from xanosmerks_b200.synth import make_weight  # noqa: E402


def main():
    out_path = sys.argv[1]
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    E, k, H, F, T = 8, 2, 1024, 2048, 160 + 16 * rank
    rng = np.random.default_rng(3)
    gate = (rng.standard_normal((E, H)) * 0.05).astype(np.float32)
    weights = {"gate": {"weight": gate}, "experts": {}}
    for e in range(E):
        weights["experts"][str(e)] = {
            wn: {"weight": GGUFTensor(make_weight("Q4_K", *shape, seed=100 + 3 * e + i), "Q4_K", shape)}
            for i, (wn, shape) in enumerate((("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F))))}
    cfg = {"num_experts": E, "num_experts_per_tok": k, "hidden_act": "silu"}
    ep = MoELayerEP(cfg, weights, rank, world)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(50 + rank)).to(torch.bfloat16).cuda()
    y = ep.forward_device(x)
    y2 = ep.forward_device(x)            # a second call reuses every buffer
    torch.cuda.synchronize()
    sizes = [None] * world
    dist.all_gather_object(sizes, T)
    tmax = max(sizes)
    pad = torch.zeros(tmax, H, device="cuda")
    pad[:T] = y
    outs = [torch.zeros(tmax, H, device="cuda") for _ in sizes]
    dist.all_gather(outs, pad)
    outs = [o[:s] for o, s in zip(outs, sizes)]
    if rank == 0:
        full = MoELayer(cfg, weights)
        rep = {"world": world, "ranks": []}
        for r in range(world):
            xr = torch.randn(sizes[r], H, generator=torch.Generator().manual_seed(50 + r)).to(torch.bfloat16).cuda()
            ref = full.forward_device(xr)
            err = float((outs[r] - ref).abs().max() / ref.abs().max())
            rep["ranks"].append({"rank": r, "rel_err": err})
        rep["repeat_equal"] = bool(torch.equal(y, y2))
        with open(out_path, "w") as f:
            json.dump(rep, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
