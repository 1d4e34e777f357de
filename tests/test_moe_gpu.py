"""GPU parity: the MoE block against the reference's MoELayer (golden) and the oracle."""

import numpy as np
import pytest
import torch

from oracle import gguf_dequant_oracle as O
from oracle.moe_oracle import ACTS, moe_forward
from tests.helpers import GEMM_TOL, rel_err
from xanosmerks_b200.moe import MoELayer
from xanosmerks_b200.ops import GGUFTensor
from xanosmerks_b200.synth import make_weight

pytestmark = pytest.mark.gpu


def _layer_from_golden(g, k):
    E, H, F = (int(v) for v in g["ehf"])
    weights = {"gate": {"weight": g["gate_w"]}, "experts": {}}
    for e in range(E):
        weights["experts"][str(e)] = {
            wn: {"weight": GGUFTensor(g[f"raw_e{e}_{wn}"], "Q4_K", shape)}
            for wn, shape in (("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F)))}
    return MoELayer({"num_experts": E, "num_experts_per_tok": k, "hidden_act": "silu"}, weights)


@pytest.mark.parametrize("k", [1, 2, 4])
def test_golden_moe(golden_moe, k):
    """Sparse top-1/top-2 and dense (k == E) against the reference's own outputs."""
    g = golden_moe
    y = _layer_from_golden(g, k)(g["x"])
    assert y.shape == g["x"].shape and y.dtype == np.float32
    assert rel_err(y, g[f"y_k{k}"]) < GEMM_TOL


def _random_moe(E, H, F, seed):
    rng = np.random.default_rng(seed)
    gate = (rng.standard_normal((E, H)) * 0.05).astype(np.float32)
    raws = {(e, wn): make_weight("Q4_K", *shape, seed=seed * 100 + 3 * e + i)
            for e in range(E) for i, (wn, shape) in enumerate((("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F))))}
    return gate, raws


@pytest.mark.parametrize("T,E,k,H,F", [(300, 8, 2, 1024, 2048), (37, 8, 2, 512, 768), (64, 4, 4, 256, 512)])
def test_moe_vs_oracle(T, E, k, H, F):
    gate, raws = _random_moe(E, H, F, seed=7)
    weights = {"gate": {"weight": gate}, "experts": {}}
    experts = []
    for e in range(E):
        weights["experts"][str(e)] = {
            wn: {"weight": GGUFTensor(raws[(e, wn)], "Q4_K", shape)}
            for wn, shape in (("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F)))}
        experts.append({wn: O.dequantize(raws[(e, wn)], "Q4_K", shape).astype(np.float32)
                        for wn, shape in (("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F)))})
    x = torch.randn(1, T, H, generator=torch.Generator().manual_seed(8)).to(torch.bfloat16)
    layer = MoELayer({"num_experts": E, "num_experts_per_tok": k}, weights)
    y = layer(x.cuda()).cpu().numpy()
    ref = moe_forward(x.float().numpy(), gate, experts, k)
    assert rel_err(y, ref) < GEMM_TOL, rel_err(y, ref)


@pytest.mark.parametrize("act", ["gelu", "relu", "identity", "swish"])
def test_moe_activations_vs_oracle(act):
    """hidden_act other than silu (apply_activation, primitives.py:52-62), and Q6_K / Q8_0 experts."""
    T, E, k, H, F = 96, 4, 2, 512, 1024
    gate, raws = _random_moe(E, H, F, seed=17)
    weights = {"gate": {"weight": gate}, "experts": {}}
    experts = []
    for e in range(E):
        weights["experts"][str(e)] = {wn: {"weight": GGUFTensor(raws[(e, wn)], "Q4_K", shape)}
                                      for wn, shape in (("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F)))}
        experts.append({wn: O.dequantize(raws[(e, wn)], "Q4_K", shape).astype(np.float32)
                        for wn, shape in (("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F)))})
    x = np.random.default_rng(18).standard_normal((1, T, H)).astype(np.float32)
    layer = MoELayer({"num_experts": E, "num_experts_per_tok": k, "hidden_act": act}, weights)
    y = layer(x)
    ref = moe_forward(x, gate, experts, k, ACTS[act])
    assert rel_err(y, ref) < GEMM_TOL, rel_err(y, ref)


@pytest.mark.parametrize("qtype", ["Q6_K", "Q8_0", "Q5_K"])
def test_moe_other_expert_types(qtype):
    T, E, k, H, F = 64, 4, 2, 2048, 2048
    rng = np.random.default_rng(19)
    gate = (rng.standard_normal((E, H)) * 0.05).astype(np.float32)
    weights = {"gate": {"weight": gate}, "experts": {}}
    experts = []
    for e in range(E):
        ew, eo = {}, {}
        for i, (wn, shape) in enumerate((("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F)))):
            raw = make_weight(qtype, *shape, seed=500 + 3 * e + i)
            ew[wn] = {"weight": GGUFTensor(raw, qtype, shape)}
            eo[wn] = O.dequantize(raw, qtype, shape).astype(np.float32)
        weights["experts"][str(e)] = ew
        experts.append(eo)
    x = rng.standard_normal((1, T, H)).astype(np.float32)
    y = MoELayer({"num_experts": E, "num_experts_per_tok": k}, weights)(x)
    ref = moe_forward(x, gate, experts, k)
    assert rel_err(y, ref) < GEMM_TOL, rel_err(y, ref)


def test_moe_mixtral_config_vs_oracle():
    """The Mixtral-shape block itself: 8 experts, top-2, 1024 bf16 tokens N(0,1), d_model 4096, FFN
    14336, Q4_K experts, router logits N(0,1) (gate rows N(0,1)/64 on unit tokens).  The oracle
    dequantizes each expert and runs its FFN on the rows routed to it in a spawned worker process;
    routing and the ordered combine are the oracle's own (moe.py:61-113)."""
    import concurrent.futures as cf
    import multiprocessing as mp

    from oracle.moe_oracle import combine, route
    from tests.moe_oracle_worker import expert_rows
    T, E, k, H, F = 1024, 8, 2, 4096, 14336
    rng = np.random.default_rng(2)
    gate = (rng.standard_normal((E, H)) / 64.0).astype(np.float32)
    raws = {(e, wn): make_weight("Q4_K", *shape, seed=3000 + 3 * e + i)
            for e in range(E) for i, (wn, shape) in enumerate((("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F))))}
    weights = {"gate": {"weight": gate}, "experts": {
        str(e): {wn: {"weight": GGUFTensor(raws[(e, wn)], "Q4_K", shape)}
                 for wn, shape in (("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F)))} for e in range(E)}}
    x = torch.randn(1, T, H, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    y = MoELayer({"num_experts": E, "num_experts_per_tok": k, "hidden_act": "silu"}, weights)(x.cuda())
    y = y.cpu().numpy().reshape(T, H)
    xf = x.float().numpy().reshape(T, H)
    routing = route(xf @ gate.T, k)
    se, sw, st, counts = routing
    starts = np.concatenate([[0], np.cumsum(counts)])
    jobs = [(raws[(e, "w1")], raws[(e, "w3")], raws[(e, "w2")], "Q4_K", H, F, xf[st[starts[e]:starts[e + 1]]],
             "silu") for e in range(E)]
    with cf.ProcessPoolExecutor(max_workers=8, mp_context=mp.get_context("spawn")) as ex:
        outs = list(ex.map(expert_rows, jobs))
    ref = combine(T, H, routing, outs)
    assert rel_err(y, ref) < GEMM_TOL, rel_err(y, ref)


def test_moe_argument_checks(golden_moe):
    g = golden_moe
    with pytest.raises(ValueError):
        _layer_from_golden(g, 0)
    with pytest.raises(ValueError):
        _layer_from_golden(g, 5)


@pytest.mark.parametrize("T,E,k,H,F,shards", [(300, 8, 2, 1024, 2048, 1), (200, 8, 2, 512, 768, 2),
                                               (96, 8, 1, 256, 512, 4)])
def test_split_entry_points_match_fused(T, E, k, H, F, shards):
    """xm_moe_dispatch -> (exchange, emulated here on one GPU for `shards`
    ranks: rows regrouped as (source rank, local expert)) -> xm_moe_experts ->
    xm_moe_combine gives the same output as xm_moe_forward."""
    import ctypes

    from xanosmerks_b200._lib import DT_BF16, check, lib
    gate, raws = _random_moe(E, H, F, seed=9)
    weights = {"gate": {"weight": gate}, "experts": {}}
    for e in range(E):
        weights["experts"][str(e)] = {
            wn: {"weight": GGUFTensor(raws[(e, wn)], "Q4_K", shape)}
            for wn, shape in (("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F)))}
    layer = MoELayer({"num_experts": E, "num_experts_per_tok": k}, weights)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(10)).to(torch.bfloat16).cuda()
    ref = layer.forward_device(x)
    st = torch.cuda.current_stream().cuda_stream
    ws = torch.zeros(lib.xm_moe_workspace_size(T, H, F, E, k), dtype=torch.uint8, device="cuda")
    send = torch.empty(T * k, H, dtype=torch.bfloat16, device="cuda")
    cnt = torch.empty(E, dtype=torch.int32, device="cuda")
    check(lib.xm_moe_dispatch(x.data_ptr(), DT_BF16, T, H, layer.gate.data_ptr(), E, k, F, send.data_ptr(),
                              cnt.data_ptr(), ws.data_ptr(), ws.numel(), st), "dispatch")
    c = cnt.cpu()
    assert int(c.sum()) == T * k
    # one rank holds all experts here; the groups are the experts themselves
    off = (torch.cumsum(c, 0) - c).to(torch.int32)
    G = E
    p1 = (ctypes.c_void_p * G)(*[layer.w1[g].data.data_ptr() for g in range(G)])
    p3 = (ctypes.c_void_p * G)(*[layer.w3[g].data.data_ptr() for g in range(G)])
    p2 = (ctypes.c_void_p * G)(*[layer.w2[g].data.data_ptr() for g in range(G)])
    rows = torch.empty(T * k, H, dtype=torch.float32, device="cuda")
    ews = torch.empty(lib.xm_moe_experts_workspace_size(T * k, H, F), dtype=torch.uint8, device="cuda")
    c_dev, off_dev = c.cuda(), off.cuda()          # kept alive: the kernels read them after the call returns
    check(lib.xm_moe_experts(send.data_ptr(), DT_BF16, T * k, H, F, G, c_dev.data_ptr(), off_dev.data_ptr(),
                             p1, p3, p2, 12, 0, int(c.max()), rows.data_ptr(), ews.data_ptr(), ews.numel(), st),
          "experts")
    out = torch.empty(T, H, dtype=torch.float32, device="cuda")
    check(lib.xm_moe_combine(rows.data_ptr(), T, H, E, k, F, ws.data_ptr(), out.data_ptr(), st), "combine")
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) < 1e-6
    assert shards >= 1
