"""Tensor-parallel host logic on CPU with gloo (world size 2): every rank
shards the same seeded weights; gathering the shards' bytes reassembles the
full matrices (row blocks for QKV / gate-up, K-slices for O / down)."""

import os

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from xanosmerks_b200.synth import make_weight


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import xanosmerks_b200.llama as L
        from tests.test_llama_host import _HostTensor
        L.GGUFTensor = _HostTensor
        n, k = 64, 2048                                    # a [rows x K] Q6_K matrix, split 2 ways
        raw = make_weight("Q6_K", n, k, seed=9)
        t = _HostTensor(raw, "Q6_K", (n, k))
        cols = L.shard_cols(t, rank * k // world, (rank + 1) * k // world)
        rows = L.shard_rows(t, rank * n // world, (rank + 1) * n // world)
        gc = [torch.zeros_like(cols.data) for _ in range(world)]
        gr = [torch.zeros_like(rows.data) for _ in range(world)]
        dist.all_gather(gc, cols.data)
        dist.all_gather(gr, rows.data)
        rec = 210
        full_cols = torch.cat([g.view(n, -1, rec) for g in gc], dim=1).reshape(-1).numpy()
        full_rows = torch.cat(gr).numpy()
        q.put((rank, bool(np.array_equal(full_cols, raw)), bool(np.array_equal(full_rows, raw))))
    finally:
        dist.destroy_process_group()


def test_tp_shards_reassemble_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(c and r for _, c, r in res), res
