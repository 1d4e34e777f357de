"""GPU parity: tensor-core dequant-GEMM against the reference's fp32 ``x @ W.T``."""

import numpy as np
import pytest
import torch

from oracle import gguf_dequant_oracle as O
from tests.helpers import GEMM_TOL, rel_err
from xanosmerks_b200 import _lib
from xanosmerks_b200.ops import GGUFTensor, LinearOp, qlinear
from xanosmerks_b200.synth import make_weight

pytestmark = pytest.mark.gpu

_W = {}


def wref(name, n, k, seed):
    key = (name, n, k, seed)
    if key not in _W:
        _W.clear()
        raw = make_weight(name, n, k, seed=seed)
        _W[key] = (raw, O.dequantize(raw, name, (n, k)).astype(np.float32))
    return _W[key]


@pytest.mark.parametrize("m,n,k", [(128, 128, 256), (200, 300, 512), (129, 176, 1024), (1000, 999, 768),
                                   (64, 11008, 4096), (512, 11008, 4096), (2048, 11008, 4096)])
def test_q4k_gemm_bf16(m, n, k):
    raw, w = wref("Q4_K", n, k, 31)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(32)).to(torch.bfloat16)
    y = qlinear(GGUFTensor(raw, "Q4_K", (n, k)), x.cuda()).cpu().numpy()
    ref = x.float().numpy() @ w.T
    e = rel_err(y, ref)
    assert e < GEMM_TOL, e
    assert e < 1e-5, e     # fp16-exact operands: only the summation order differs


def test_q4k_gemm_fp32_bias_and_row_scales():
    m, n, k = 300, 512, 1024
    raw, w = wref("Q4_K", n, k, 41)
    x = np.random.default_rng(42).standard_normal((m, k)).astype(np.float32)
    x[0] *= 1e5          # rows beyond fp16's range and far below it: the per-row scale keeps them exact
    x[1] *= 1e-6
    b = np.random.default_rng(43).standard_normal(n).astype(np.float32)
    y = LinearOp(GGUFTensor(raw, "Q4_K", (n, k)), b).forward(x)
    ref = x @ w.T + b
    for r in (0, 1):
        assert rel_err(y[r], ref[r]) < GEMM_TOL
    assert rel_err(y, ref) < GEMM_TOL


def test_q4k_gemm_matches_gemv_rows():
    """The GEMM and the decode GEMV agree on the same rows."""
    m, n, k = 96, 640, 4096
    raw, w = wref("Q4_K", n, k, 51)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(52)).to(torch.bfloat16).cuda()
    W = GGUFTensor(raw, "Q4_K", (n, k))
    y_gemm = qlinear(W, x).cpu().numpy()
    y_gemv = np.concatenate([qlinear(W, x[i:i + 8]).cpu().numpy() for i in range(0, m, 8)])
    assert rel_err(y_gemm, y_gemv) < 1e-3


def test_qgemm_rejects_bad_arguments():
    L = _lib.lib
    assert L.xm_qgemm(14, None, 0, 4, 256, None, 0, 64, None, None, None, 0, None) == _lib.XM_ERR_UNSUPPORTED
    assert L.xm_qgemm(12, None, 0, 4, 300, None, 0, 64, None, None, None, 0, None) == _lib.XM_ERR_INVALID
