"""GPU parity: the MoE block against the reference's MoELayer (golden) and the oracle."""

import numpy as np
import pytest
import torch

from oracle import gguf_dequant_oracle as O
from oracle.moe_oracle import moe_forward
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


def test_moe_argument_checks(golden_moe):
    g = golden_moe
    with pytest.raises(ValueError):
        _layer_from_golden(g, 0)
    with pytest.raises(ValueError):
        _layer_from_golden(g, 5)
