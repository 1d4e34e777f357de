"""Expert-parallel host logic on CPU with gloo (world size 2): the exchange in
``xanosmerks_b200.moe.ep_exchange`` (counts, rows out, (source rank, local
expert) groups, rows back) driven by the oracle's routing and expert FFNs
reproduces the single-process MoE block (moe.py:54-115) on every rank."""

import os

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, F, E, K, T = 64, 96, 4, 2, 37


def _weights():
    rng = np.random.default_rng(11)
    gate = rng.standard_normal((E, H)).astype(np.float32)
    experts = [{"w1": (rng.standard_normal((F, H)) * 0.1).astype(np.float32),
                "w3": (rng.standard_normal((F, H)) * 0.1).astype(np.float32),
                "w2": (rng.standard_normal((H, F)) * 0.1).astype(np.float32)} for _ in range(E)]
    return gate, experts


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.moe_oracle import moe_forward, route, silu
        from xanosmerks_b200.moe import ep_exchange
        gate, experts = _weights()
        e_local = E // world
        x = np.random.default_rng(100 + rank).standard_normal((T, H)).astype(np.float32)
        # dispatch: routed rows in ascending expert order and rows per expert
        se, sw, st, counts = route(x @ gate.T, K)
        send = torch.from_numpy(np.ascontiguousarray(x[st]))
        cnt = torch.from_numpy(np.asarray(counts, dtype=np.int32))

        def run_experts(recv, rc, off):
            r = recv.numpy()
            rows = np.zeros_like(r)
            for g in range(world * e_local):          # g = (source rank, local expert)
                e = rank * e_local + g % e_local
                a, b = int(off[g]), int(off[g] + rc[g])
                xs = r[a:b]
                rows[a:b] = (silu(xs @ experts[e]["w1"].T) * (xs @ experts[e]["w3"].T)) @ experts[e]["w2"].T
            return torch.from_numpy(rows)

        back = ep_exchange(send, cnt, world, e_local, dist.group.WORLD, run_experts).numpy()
        out = np.zeros_like(x)
        for j in range(len(st)):                      # combine in ascending expert order, as moe.py does
            out[st[j]] += back[j] * sw[j]
        ref = moe_forward(x[None], gate, experts, K)[0]
        err = float(np.abs(out - ref).max() / np.abs(ref).max())
        q.put((rank, err, int(sum(counts))))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e), -1))
    finally:
        dist.destroy_process_group()


def test_ep_exchange_matches_single_process_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, 29000 + os.getpid() % 1000
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(60)
    for rank, err, n in res:
        assert not isinstance(err, str), err
        assert n == T * K
        assert err < 1e-6, (rank, err)
