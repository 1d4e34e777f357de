"""GPU parity: the generic integer-dot GEMV (Q4_K, Q5_K, Q6_K, Q8_0 at any row
length) and the fused prologue / residual forms of ``xm_qgemv_ex``, against
the reference's fp32 ``x @ W.T`` on its fp16 weights (ops.py:62-67), its
``FusedRMSNormLinearOp`` (ops.py:107-123) and its MLP down projection on
``swiglu(gate, up)`` (forward.py:97-101)."""

import numpy as np
import pytest
import torch

from oracle import gguf_dequant_oracle as O
from tests.helpers import GEMV_TOL, rel_err
from xanosmerks_b200._lib import DT_F32, PRO_NONE, PRO_RMSNORM, PRO_SWIGLU, check, lib
from xanosmerks_b200.ops import GGUFTensor, qlinear
from xanosmerks_b200.synth import make_weight

pytestmark = pytest.mark.gpu

_W = {}


def weight(name, n, k, seed):
    key = (name, n, k, seed)
    if key not in _W:
        if len(_W) > 3:
            _W.clear()
        raw = make_weight(name, n, k, seed=seed)
        _W[key] = (raw, O.dequantize(raw, name, (n, k)).astype(np.float32))
    return _W[key]


def qgemv_ex(W, x, m, x_stride, prologue=PRO_NONE, norm=None, y=None, accumulate=False, eps=1e-5):
    n, k = W.shape
    if y is None:
        y = torch.zeros(m, n, dtype=torch.float32, device="cuda")
    ws = torch.zeros(lib.xm_qgemv_workspace_size(k, m) + 256, dtype=torch.uint8, device="cuda")
    check(lib.xm_qgemv_ex(W.qtype.type_id, W.data.data_ptr(), W.nbytes, n, k, x.data_ptr(), DT_F32, m, x_stride,
                          prologue, norm.data_ptr() if norm is not None else None, eps, None, y.data_ptr(),
                          1 if accumulate else 0, ws.data_ptr(), ws.numel(),
                          torch.cuda.current_stream().cuda_stream), "qgemv_ex")
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("name", ["Q4_K", "Q5_K", "Q6_K", "Q8_0"])
@pytest.mark.parametrize("n,k", [(4096, 4096), (4096, 14336), (14336, 4096)])
@pytest.mark.parametrize("m", [1, 4])
def test_decode_shapes(name, n, k, m):
    """The Q6_K / Q5_K decode shapes at batch 1 and 4 (and the same for Q4_K, Q8_0)."""
    raw, wf = weight(name, n, k, 11)
    x = np.random.default_rng(12).standard_normal((m, k)).astype(np.float32)
    y = qlinear(GGUFTensor(raw, name, (n, k)), torch.from_numpy(x).cuda()).cpu().numpy()
    assert rel_err(y, x @ wf.T) < GEMV_TOL


@pytest.mark.parametrize("name,n,k", [("Q6_K", 1000, 1792), ("Q6_K", 37, 512), ("Q5_K", 999, 2048),
                                      ("Q8_0", 513, 128), ("Q8_0", 77, 1792), ("Q4_K", 301, 14336),
                                      ("Q6_K", 5, 16384), ("Q5_K", 3, 8192)])
@pytest.mark.parametrize("m", [1, 3, 8])
def test_ragged_shapes(name, n, k, m):
    """Row counts that leave partial chunks, rows whose byte length is not a
    multiple of 16 (Q6_K K=1792: 1470 B), parts P = 1, 2, 4."""
    raw, wf = weight(name, n, k, 13)
    x = np.random.default_rng(14).standard_normal((m, k)).astype(np.float32)
    y = qlinear(GGUFTensor(raw, name, (n, k)), torch.from_numpy(x).cuda()).cpu().numpy()
    assert rel_err(y, x @ wf.T) < GEMV_TOL


def test_integer_matches_exact_path():
    """Same weights through the integer path and the fp16-exact path."""
    for name in ("Q5_K", "Q6_K", "Q8_0"):
        raw, _ = weight(name, 640, 4096, 15)
        W = GGUFTensor(raw, name, (640, 4096))
        x = torch.randn(2, 4096, device="cuda")
        a = qlinear(W, x).cpu().numpy()
        b = qlinear(W, x, exact=True).cpu().numpy()
        assert rel_err(a, b) < GEMV_TOL, name


def rms(x, w, eps=1e-5):
    return (x / np.sqrt(np.mean(x ** 2, axis=-1, keepdims=True) + eps)) * w


def silu(x):
    return x / (1.0 + np.exp(-x))


@pytest.mark.parametrize("name,n,k,m", [("Q4_K", 6144, 4096, 1), ("Q4_K", 1024, 4096, 3), ("Q6_K", 4096, 4096, 1),
                                        ("Q6_K", 2000, 4096, 8), ("Q5_K", 512, 2048, 2)])
def test_rmsnorm_prologue(name, n, k, m):
    """FusedRMSNormLinearOp: rms_norm(x) * w then @ W.T (the Q4_K single-row
    K = 4096 case runs the norm inside the GEMV kernel)."""
    raw, wf = weight(name, n, k, 21)
    rng = np.random.default_rng(22)
    x = (3.0 * rng.standard_normal((m, k))).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    W = GGUFTensor(raw, name, (n, k))
    y = qgemv_ex(W, torch.from_numpy(x).cuda(), m, k, PRO_RMSNORM, torch.from_numpy(nw).cuda()).cpu().numpy()
    assert rel_err(y, rms(x, nw) @ wf.T) < GEMV_TOL


@pytest.mark.parametrize("name,n,k,m", [("Q6_K", 4096, 14336, 1), ("Q6_K", 4096, 14336, 2), ("Q4_K", 512, 4096, 1),
                                        ("Q6_K", 300, 1792, 4)])
def test_swiglu_prologue_and_residual(name, n, k, m):
    """h += swiglu(gate, up) @ W_down.T with x rows holding [gate | up]."""
    raw, wf = weight(name, n, k, 31)
    rng = np.random.default_rng(32)
    gu = (2.0 * rng.standard_normal((m, 2 * k))).astype(np.float32)
    h0 = rng.standard_normal((m, n)).astype(np.float32)
    W = GGUFTensor(raw, name, (n, k))
    y = torch.from_numpy(h0.copy()).cuda()
    qgemv_ex(W, torch.from_numpy(gu).cuda(), m, 2 * k, PRO_SWIGLU, y=y, accumulate=True)
    ref = h0 + (silu(gu[:, :k]) * gu[:, k:]) @ wf.T
    assert rel_err(y.cpu().numpy(), ref) < GEMV_TOL


@pytest.mark.parametrize("name,k", [("Q4_K", 4096), ("Q6_K", 4096), ("Q4_K", 1024)])
def test_accumulate_plain(name, k):
    raw, wf = weight(name, 700, k, 41)
    rng = np.random.default_rng(42)
    x = rng.standard_normal((1, k)).astype(np.float32)
    h0 = rng.standard_normal((1, 700)).astype(np.float32)
    y = torch.from_numpy(h0.copy()).cuda()
    qgemv_ex(GGUFTensor(raw, name, (700, k)), torch.from_numpy(x).cuda(), 1, k, y=y, accumulate=True)
    assert rel_err(y.cpu().numpy(), h0 + x @ wf.T) < GEMV_TOL


def test_prologue_needs_integer_path():
    """Types without an integer-dot path take no prologue (NotImplementedError)."""
    raw = make_weight("Q3_K", 64, 256, seed=1)
    W = GGUFTensor(raw, "Q3_K", (64, 256))
    x = torch.randn(1, 256, device="cuda")
    with pytest.raises(NotImplementedError):
        qgemv_ex(W, x, 1, 256, PRO_RMSNORM, torch.ones(256, device="cuda"))
    assert lib.xm_device_status(1) == 0


@pytest.mark.parametrize("n,k", [(4096, 4096), (6144, 4096), (1000, 2048), (37, 512), (28672, 4096), (300, 8192)])
@pytest.mark.parametrize("m", [2, 3, 4, 5, 8])
def test_q4k_tensor_core_batch(n, k, m):
    """Q4_K with 2..8 activation rows runs on the tensor cores (integer MMA,
    one scale per activation row); plain, RMSNorm prologue and residual add."""
    raw, wf = weight("Q4_K", n, k, 51)
    rng = np.random.default_rng(52)
    x = (2.0 * rng.standard_normal((m, k))).astype(np.float32)
    W = GGUFTensor(raw, "Q4_K", (n, k))
    y = qlinear(W, torch.from_numpy(x).cuda()).cpu().numpy()
    assert rel_err(y, x @ wf.T) < GEMV_TOL
    nw = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    h0 = rng.standard_normal((m, n)).astype(np.float32)
    yy = torch.from_numpy(h0.copy()).cuda()
    qgemv_ex(W, torch.from_numpy(x).cuda(), m, k, PRO_RMSNORM, torch.from_numpy(nw).cuda(), y=yy, accumulate=True)
    assert rel_err(yy.cpu().numpy(), h0 + rms(x, nw) @ wf.T) < GEMV_TOL
    assert lib.xm_device_status(0) == 0


def test_q4k_tensor_core_swiglu():
    raw, wf = weight("Q4_K", 2048, 4096, 53)
    rng = np.random.default_rng(54)
    gu = (2.0 * rng.standard_normal((6, 8192))).astype(np.float32)
    y = qgemv_ex(GGUFTensor(raw, "Q4_K", (2048, 4096)), torch.from_numpy(gu).cuda(), 6, 8192, PRO_SWIGLU)
    ref = (silu(gu[:, :4096]) * gu[:, 4096:]) @ wf.T
    assert rel_err(y.cpu().numpy(), ref) < GEMV_TOL
