"""GPU parity: fused dequant-GEMV against the reference's fp32 ``x @ W.T`` on its fp16 weights."""

import numpy as np
import pytest
import torch

from oracle import gguf_dequant_oracle as O
from tests.helpers import GEMV_TOL, rel_err
from xanosmerks_b200.ops import GGUFTensor, LinearOp, qlinear
from xanosmerks_b200.synth import QK, RECORD, make_weight

pytestmark = pytest.mark.gpu


_WCACHE = {}


def ref_y(raw, name, n, k, x):
    key = (name, n, k, raw[:64].tobytes(), raw.size)
    if key not in _WCACHE:
        _WCACHE.clear()
        _WCACHE[key] = O.dequantize(raw, name, (n, k)).astype(np.float32)
    return np.asarray(x, np.float32) @ _WCACHE[key].T


def test_golden_linear(golden_linear):
    g = golden_linear
    for name in ("Q4_K", "Q6_K", "Q8_0", "Q5_K", "Q4_0"):
        n, k = (int(v) for v in g[f"{name}_nk"])
        W = GGUFTensor(g[f"{name}_raw"], name, (n, k))
        for m in (1, 3, 8):
            y = LinearOp(W).forward(g[f"{name}_m{m}_x"])
            assert y.dtype == np.float32
            assert rel_err(y, g[f"{name}_m{m}_y"]) < GEMV_TOL, (name, m)
        y = LinearOp(W, g[f"{name}_bias_b"]).forward(g[f"{name}_bias_x"])
        assert y.shape == g[f"{name}_bias_y"].shape
        assert rel_err(y, g[f"{name}_bias_y"]) < GEMV_TOL


@pytest.mark.parametrize("name", list(RECORD))
@pytest.mark.parametrize("m", [1, 4, 8])
def test_exact_path_all_types(name, m):
    n, k = 96, 1024
    raw = make_weight(name, n, k, seed=5)
    x = np.random.default_rng(6).standard_normal((m, k)).astype(np.float32)
    W = GGUFTensor(raw, name, (n, k))
    y = qlinear(W, torch.from_numpy(x).cuda(), exact=True).cpu().numpy()
    assert rel_err(y, ref_y(raw, name, n, k, x)) < 1e-5     # same fp16 weights; only summation order differs


@pytest.mark.parametrize("n,k", [(11008, 4096), (4096, 14336), (37, 512), (1, 256), (4099, 2816)])
@pytest.mark.parametrize("xdt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8])
def test_q4k_integer_path(m, xdt, n, k):
    raw = make_weight("Q4_K", n, k, seed=11)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(12)).to(xdt)
    W = GGUFTensor(raw, "Q4_K", (n, k))
    y = qlinear(W, x.cuda()).cpu().numpy()
    e = rel_err(y, ref_y(raw, "Q4_K", n, k, x.float().numpy()))
    assert e < GEMV_TOL, e


def test_q4k_bias_and_batch_dims():
    n, k = 300, 512
    raw = make_weight("Q4_K", n, k, seed=1)
    x = np.random.default_rng(2).standard_normal((2, 3, k)).astype(np.float32)
    b = np.random.default_rng(3).standard_normal(n).astype(np.float32)
    y = LinearOp(GGUFTensor(raw, "Q4_K", (n, k)), b).forward(x)
    assert y.shape == (2, 3, n)
    assert rel_err(y, ref_y(raw, "Q4_K", n, k, x) + b) < GEMV_TOL
