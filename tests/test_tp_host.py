"""Tensor-parallel host logic on CPU with gloo (world size 2): every rank
shards the same seeded weights; gathering the shards' bytes reassembles the
full matrices (row blocks for QKV / gate-up, K-slices for O / down); and one
layer's projections computed from each rank's shard, with the row-parallel
partial sums all-reduced, equal the unsharded layer."""

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


def _forward_worker(rank, world, port, q):
    """One decoder layer's projections, tensor-parallel as LlamaWeights.from_full shards them: QKV and
    gate/up column-parallel (this rank's heads / FFN columns), O and down row-parallel over K with the
    partial sums all-reduced (gloo here, the NVLink all-reduce or NCCL on GPUs).  Each rank decodes its
    own shard's bytes with the oracle; the result must equal the unsharded layer on every rank."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import xanosmerks_b200.llama as L
        from oracle import gguf_dequant_oracle as O
        from oracle.llama_oracle import rms_norm, silu
        from tests.test_llama_host import _HostTensor
        L.GGUFTensor = _HostTensor
        cfg = L.LlamaConfig(num_layers=1, hidden_size=512, num_heads=8, num_kv_heads=4, head_dim=64,
                            intermediate_size=1024, vocab_size=256)
        D, F, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
        shapes = {"wq": (cfg.num_heads * hd, D), "wk": (cfg.num_kv_heads * hd, D), "wv": (cfg.num_kv_heads * hd, D),
                  "wo": (D, cfg.num_heads * hd), "wg": (F, D), "wu": (F, D), "wd": (D, F)}
        types = {"wq": "Q4_K", "wk": "Q4_K", "wv": "Q4_K", "wo": "Q4_K", "wg": "Q4_K", "wu": "Q4_K", "wd": "Q6_K"}
        raws = {n: make_weight(types[n], *shapes[n], seed=40 + i) for i, n in enumerate(shapes)}
        rng = np.random.default_rng(41)
        n1 = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
        n2 = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
        layer = {n: _HostTensor(raws[n], types[n], shapes[n]) for n in shapes}
        layer.update(n1=torch.from_numpy(n1), n2=torch.from_numpy(n2))
        full = {"embed": None, "layers": [layer], "norm": None, "output": None}
        w = L.LlamaWeights.from_full(cfg, full, rank, world).layers[0]

        def deq(t):
            return O.dequantize(t.data.numpy().tobytes(), t.qtype.name, t.shape).astype(np.float32)

        h = rng.standard_normal((3, D)).astype(np.float32)
        attn = rng.standard_normal((3, cfg.num_heads * hd)).astype(np.float32)
        hq_l, f_l = cfg.num_heads // world, F // world
        # O projection: this rank's heads' columns of attn against its K-slice, summed over ranks
        part = attn[:, rank * hq_l * hd:(rank + 1) * hq_l * hd] @ deq(w["o"]).T
        tp = torch.from_numpy(np.ascontiguousarray(part))
        dist.all_reduce(tp)
        o_full = attn @ O.dequantize(raws["wo"], "Q4_K", shapes["wo"]).astype(np.float32).T
        ok_o = float(np.abs(tp.numpy() - o_full).max() / np.abs(o_full).max())
        # MLP: gate/up rows of this rank, SwiGLU locally, down's matching K-slice, all-reduce
        gu = rms_norm(h, n2, cfg.norm_eps) @ deq(w["gate_up"]).T
        hid = silu(gu[:, :f_l]) * gu[:, f_l:]
        tm = torch.from_numpy(np.ascontiguousarray(hid @ deq(w["down"]).T))
        dist.all_reduce(tm)
        wg, wu = (O.dequantize(raws[n], "Q4_K", shapes[n]).astype(np.float32) for n in ("wg", "wu"))
        wd = O.dequantize(raws["wd"], "Q6_K", shapes["wd"]).astype(np.float32)
        hn = rms_norm(h, n2, cfg.norm_eps)
        mlp_full = (silu(hn @ wg.T) * (hn @ wu.T)) @ wd.T
        ok_m = float(np.abs(tm.numpy() - mlp_full).max() / np.abs(mlp_full).max())
        # QKV: this rank's q heads then k, v heads, against the same rows of the full projections
        qkv = rms_norm(h, n1, cfg.norm_eps) @ deq(w["qkv"]).T
        hk_l = cfg.num_kv_heads // world
        hn1 = rms_norm(h, n1, cfg.norm_eps)
        q_full = hn1 @ O.dequantize(raws["wq"], "Q4_K", shapes["wq"]).astype(np.float32).T
        k_full = hn1 @ O.dequantize(raws["wk"], "Q4_K", shapes["wk"]).astype(np.float32).T
        want = np.concatenate([q_full[:, rank * hq_l * hd:(rank + 1) * hq_l * hd],
                               k_full[:, rank * hk_l * hd:(rank + 1) * hk_l * hd]], axis=1)
        ok_q = float(np.abs(qkv[:, :want.shape[1]] - want).max() / np.abs(want).max())
        q.put((rank, ok_o, ok_m, ok_q))
    finally:
        dist.destroy_process_group()


def test_tp_layer_partial_sums_allreduce_match_unsharded_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_forward_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, eo, em, eq in res:
        assert eo < 1e-5 and em < 1e-5 and eq < 1e-6, (rank, eo, em, eq)
