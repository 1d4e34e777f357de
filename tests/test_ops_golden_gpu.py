"""GPU parity of the drop-in operator classes against outputs of the reference itself
(tests/golden/golden_linear.npz, written by make_golden.py from ops.py / primitives.py):

* ``FusedRMSNormLinearOp(norm_weight, W).forward(x)`` (ops.py:107-123), for quantized
  weights (norm fused into the GEMV prologue, or a separate norm kernel where the type
  has no fused path) and for the dense weight the reference itself takes;
* the SwiGLU MLP ``swiglu(x @ Wg.T, x @ Wu.T) @ Wd.T`` (forward.py:93-103,
  primitives.py:42-44) through the fused down-projection prologue;
* ``LinearOp`` with a dense weight, as the reference's own health check builds it
  (``LinearOp(np.eye(4))``, defaults.py:109-117).
"""

import numpy as np
import pytest
import torch

from tests.helpers import GEMM_TOL, GEMV_TOL, rel_err
from xanosmerks_b200._lib import PRO_SWIGLU
from xanosmerks_b200.ops import FusedRMSNormLinearOp, GGUFTensor, LinearOp, qlinear

pytestmark = pytest.mark.gpu

NAMES = ["Q4_K", "Q6_K", "Q8_0", "Q5_K", "Q4_0"]


def _w(g, name):
    n, k = (int(v) for v in g[f"{name}_nk"])
    return GGUFTensor(g[f"{name}_raw"], name, (n, k)), n, k


@pytest.mark.parametrize("name", NAMES)
def test_fused_rmsnorm_linear_golden(golden_linear, name):
    g = golden_linear
    W, n, k = _w(g, name)
    op = FusedRMSNormLinearOp(g[f"{name}_rms_nw"], W)
    x = g[f"{name}_bias_x"]                           # (2, 3, k): 6 rows -> the decode path
    y = op.forward(x)
    assert y.shape == (2, 3, n) and y.dtype == np.float32
    assert rel_err(y, g[f"{name}_rms_y"]) < GEMV_TOL, rel_err(y, g[f"{name}_rms_y"])
    # the same rows as a CUDA tensor, and many rows (tensor-core GEMM where the type has one)
    yd = op.forward(torch.from_numpy(x).cuda()).cpu().numpy()
    assert rel_err(yd, g[f"{name}_rms_y"]) < GEMV_TOL
    xr = np.concatenate([x.reshape(-1, k)] * 20)     # 120 rows
    yr = op.forward(xr)
    assert rel_err(yr, np.concatenate([g[f"{name}_rms_y"].reshape(-1, n)] * 20)) < GEMM_TOL


@pytest.mark.parametrize("name", ["Q4_K", "Q8_0"])
def test_fused_rmsnorm_linear_dense_weight_golden(golden_linear, name):
    """The reference's own form: a dense fp32 weight (the dequantized matrix)."""
    g = golden_linear
    W, n, k = _w(g, name)
    dense = W.dequantize().float().cpu().numpy()
    y = FusedRMSNormLinearOp(g[f"{name}_rms_nw"], dense).forward(g[f"{name}_bias_x"])
    assert rel_err(y, g[f"{name}_rms_y"]) < 1e-5


def test_swiglu_mlp_golden(golden_linear):
    """gate/up Q4_K (one row-concatenated weight), down Q6_K with the SwiGLU prologue."""
    g = golden_linear
    h, f = (int(v) for v in g["mlp_hf"])
    gu = GGUFTensor(np.concatenate([g["mlp_gate_raw"], g["mlp_up_raw"]]), "Q4_K", (2 * f, h))
    down = GGUFTensor(g["mlp_down_raw"], "Q6_K", (h, f))
    x = torch.from_numpy(g["mlp_x"]).cuda()                  # (1, 4, h)
    a = qlinear(gu, x)                                         # (1, 4, 2f): gate then up
    y = qlinear(down, a, prologue=PRO_SWIGLU).cpu().numpy()
    assert y.shape == g["mlp_y"].shape
    assert rel_err(y, g["mlp_y"]) < GEMV_TOL, rel_err(y, g["mlp_y"])
    # many rows: the same composition on the tensor-core GEMM
    xr = x.reshape(-1, h).repeat(40, 1)                        # 160 rows
    yr = qlinear(down, qlinear(gu, xr), prologue=PRO_SWIGLU).cpu().numpy()
    assert rel_err(yr, np.tile(g["mlp_y"].reshape(-1, h), (40, 1))) < GEMM_TOL


def test_linear_op_dense_weight():
    eye = LinearOp(np.eye(4, dtype=np.float32))
    x = np.arange(8, dtype=np.float32).reshape(2, 4)
    assert np.array_equal(eye.forward(x), x)
    rng = np.random.default_rng(5)
    w = rng.standard_normal((33, 64)).astype(np.float32)
    b = rng.standard_normal(33).astype(np.float32)
    xs = rng.standard_normal((3, 5, 64)).astype(np.float32)
    y = LinearOp(w, b).forward(xs)
    assert y.shape == (3, 5, 33)
    assert rel_err(y, xs @ w.T + b) < 1e-6


def test_linear_op_golden_through_host_staging(golden_linear):
    """The host-input path (pinned staging buffers, one synchronisation, device error word read
    behind the result) on the reference's LinearOp outputs, twice with the same and with a new
    shape (the staging buffers are reused, then rebuilt)."""
    g = golden_linear
    W, n, k = _w(g, "Q4_K")
    op = LinearOp(W, g["Q4_K_bias_b"])
    for _ in range(2):
        y = op.forward(g["Q4_K_bias_x"])
        assert rel_err(y, g["Q4_K_bias_y"]) < GEMV_TOL
    y1 = LinearOp(W).forward(g["Q4_K_m1_x"])
    assert rel_err(y1, g["Q4_K_m1_y"]) < GEMV_TOL
    yt = op.forward(torch.from_numpy(g["Q4_K_bias_x"]))      # host torch tensor in -> host tensor out
    assert isinstance(yt, torch.Tensor) and not yt.is_cuda
    assert rel_err(yt.numpy(), g["Q4_K_bias_y"]) < GEMV_TOL
