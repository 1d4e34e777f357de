"""GPU parity: tensor-core dequant-GEMM against the reference's fp32 ``x @ W.T``
(ops.py:62-67) on the weights the reference dequantizes (gguf_dequant.py:25-455),
for every block type, with the RMSNorm / SwiGLU prologues and the residual add
of ``xm_qgemm_ex`` (ops.py:107-123, forward.py:97-101, :116)."""

import numpy as np
import pytest
import torch

from oracle import gguf_dequant_oracle as O
from tests.helpers import GEMM_TOL, rel_err
from xanosmerks_b200 import _lib
from xanosmerks_b200.ops import GGUFTensor, LinearOp, gemm_supported, qlinear
from xanosmerks_b200.qtypes import QUANT_NAMES, normalize
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
    for plain in (0, 1, 30, 16, 99):          # F32, F16, BF16, IQ2_XXS, unknown
        assert L.xm_qgemm(plain, None, 0, 4, 256, None, 0, 64, None, None, None, 0, None) == _lib.XM_ERR_UNSUPPORTED
    assert L.xm_qgemm(12, None, 0, 4, 300, None, 0, 64, None, None, None, 0, None) == _lib.XM_ERR_INVALID
    assert L.xm_qgemm(14, None, 0, 4, 256, None, 0, 64, None, None, None, 0, None) == _lib.XM_ERR_INVALID  # short


def _gemm(W, x, prologue=_lib.PRO_NONE, norm=None, y=None, accumulate=False, eps=1e-5, bias=None, split=False):
    """xm_qgemm_ex on a CUDA activation (fp32 rows of k, or 2k for SwiGLU); `split` sizes the
    workspace for split-K partial planes."""
    n, k = W.shape
    m = x.shape[0]
    if y is None:
        y = torch.zeros(m, n, dtype=torch.float32, device="cuda")
    wsz = _lib.lib.xm_qgemm_workspace_size_n(m, n, k) if split else _lib.lib.xm_qgemm_workspace_size(m, k)
    ws = torch.empty(wsz, dtype=torch.uint8, device="cuda")
    dt = {torch.float32: _lib.DT_F32, torch.bfloat16: _lib.DT_BF16, torch.float16: _lib.DT_F16}[x.dtype]
    _lib.check(_lib.lib.xm_qgemm_ex(W.qtype.type_id, W.data.data_ptr(), W.nbytes, n, k, x.data_ptr(), dt, m,
                                    x.shape[1], prologue, norm.data_ptr() if norm is not None else None, eps,
                                    bias.data_ptr() if bias is not None else None, y.data_ptr(),
                                    1 if accumulate else 0, ws.data_ptr(), ws.numel(),
                                    torch.cuda.current_stream().cuda_stream), "qgemm_ex")
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("name", QUANT_NAMES)
@pytest.mark.parametrize("m,n,k", [(300, 320, 2048), (77, 96, 256)])
def test_gemm_every_block_type(name, m, n, k):
    """Each of the twelve block types on the tensor cores (the generic decode for all but Q4_K), with
    the column start rounded down to 16 bytes for records whose 256-wide column is not 16-byte sized."""
    qt = normalize(name)
    if not gemm_supported(qt, k):
        pytest.skip(f"{name} rows of {k} are not whole 16-byte units")
    raw, w = wref(name, n, k, 61)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(62)).to(torch.bfloat16)
    y = _gemm(GGUFTensor(raw, name, (n, k)), x.cuda()).cpu().numpy()
    ref = x.float().numpy() @ w.T
    e = rel_err(y, ref)
    assert e < 1e-5, (name, e)       # fp16-exact operands: only the summation order differs


@pytest.mark.parametrize("name,m,n,k", [("Q6_K", 512, 4096, 14336), ("Q5_K", 512, 4096, 4096),
                                        ("Q6_K", 300, 4096, 4096), ("Q5_K", 200, 14336, 4096),
                                        ("Q8_0", 256, 4096, 4096)])
def test_gemm_config_shapes(name, m, n, k):
    """The decode / prefill shapes of the Llama config: Q6_K down projection (K = 14336) and the
    Q5_K / Q8_0 matrices, against the oracle."""
    raw, w = wref(name, n, k, 71)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(72)).to(torch.bfloat16)
    y = qlinear(GGUFTensor(raw, name, (n, k)), x.cuda()).cpu().numpy()
    ref = x.float().numpy() @ w.T
    # fp16-exact operands; the fp32 accumulation-order difference grows with K
    assert rel_err(y, ref) < 1e-5 * max(1.0, k / 4096), rel_err(y, ref)


@pytest.mark.parametrize("name", ["Q4_K", "Q6_K", "Q4_0"])
def test_gemm_rmsnorm_prologue_bias(name):
    """FusedRMSNormLinearOp for many rows (ops.py:107-123): the norm in the activation preparation."""
    m, n, k = 200, 256, 2048
    raw, w = wref(name, n, k, 81)
    rng = np.random.default_rng(82)
    x = rng.standard_normal((m, k)).astype(np.float32) * 3.0
    nw = (1 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    y = _gemm(GGUFTensor(raw, name, (n, k)), torch.from_numpy(x).cuda(), _lib.PRO_RMSNORM,
              torch.from_numpy(nw).cuda(), bias=torch.from_numpy(b).cuda()).cpu().numpy()
    rms = np.sqrt(np.mean(x ** 2, axis=-1, keepdims=True) + 1e-5)
    ref = ((x / rms) * nw) @ w.T + b
    assert rel_err(y, ref) < GEMM_TOL, rel_err(y, ref)


@pytest.mark.parametrize("name", ["Q6_K", "Q5_K"])
def test_gemm_swiglu_prologue_accumulate(name):
    """The prefill MLP down projection with its residual add: h += swiglu(gate, up) @ W_down.T
    (forward.py:97-101, :116), rows of x holding gate then up."""
    m, n, k = 160, 512, 2048
    raw, w = wref(name, n, k, 91)
    rng = np.random.default_rng(92)
    gu = rng.standard_normal((m, 2 * k)).astype(np.float32)
    h0 = rng.standard_normal((m, n)).astype(np.float32)
    y = torch.from_numpy(h0.copy()).cuda()
    _gemm(GGUFTensor(raw, name, (n, k)), torch.from_numpy(gu).cuda(), _lib.PRO_SWIGLU, y=y, accumulate=True)
    g, u = gu[:, :k], gu[:, k:]
    ref = h0 + ((g / (1.0 + np.exp(-g))) * u) @ w.T
    assert rel_err(y.cpu().numpy(), ref) < GEMM_TOL


@pytest.mark.parametrize("name", ["Q4_K", "Q8_0", "Q6_K"])
@pytest.mark.parametrize("accumulate", [False, True])
def test_gemm_many_tiles_per_pair(name, accumulate):
    """Several 256-token tiles per CTA pair (5 token tiles x 36 feature tiles over 74 pairs), so the
    accumulator is drained and refilled between tiles inside one launch: with bias, and as the
    residual add (y += x W^T + b).  Q8_0 records stage with fewer pipeline stages."""
    m, n, k = 1200, 9216, 2048
    raw, w = wref(name, n, k, 97)
    rng = np.random.default_rng(98)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(99)).to(torch.bfloat16)   # exact in fp16
    b = rng.standard_normal(n).astype(np.float32)
    h0 = rng.standard_normal((m, n)).astype(np.float32) if accumulate else np.zeros((m, n), np.float32)
    y = torch.from_numpy(h0.copy()).cuda()
    _gemm(GGUFTensor(raw, name, (n, k)), x.cuda(), y=y, accumulate=accumulate, bias=torch.from_numpy(b).cuda())
    ref = h0 + x.float().numpy() @ w.T + b
    assert rel_err(y.cpu().numpy(), ref) < 1e-5, rel_err(y.cpu().numpy(), ref)


def test_gemm_row_pitch_not_16_bytes_falls_back_to_gemv():
    """Q6_K rows of 1792 (a tensor-parallel K-slice of 14336 over 8 ranks) are 1470 bytes: the
    GEMM reports UNSUPPORTED and qlinear multiplies them on the GEMV in groups of 8 rows."""
    m, n, k = 40, 300, 1792
    raw, w = wref("Q6_K", n, k, 95)
    W = GGUFTensor(raw, "Q6_K", (n, k))
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(96)).to(torch.bfloat16).cuda()
    ws = torch.empty(_lib.lib.xm_qgemm_workspace_size(m, k), dtype=torch.uint8, device="cuda")
    y = torch.empty(m, n, dtype=torch.float32, device="cuda")
    st = _lib.lib.xm_qgemm(14, W.data.data_ptr(), W.nbytes, n, k, x.data_ptr(), _lib.DT_BF16, m, None, y.data_ptr(),
                           ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.XM_ERR_UNSUPPORTED and b"multiple of 16" in _lib.lib.xm_last_error()
    yq = qlinear(W, x).cpu().numpy()
    assert rel_err(yq, x.float().cpu().numpy() @ w.T) < 1e-3


@pytest.mark.parametrize("name,m,n,k", [("Q6_K", 64, 4096, 14336), ("Q4_K", 200, 4096, 4096),
                                        ("Q8_0", 96, 1024, 2048), ("Q4_K", 37, 11008, 4096)])
@pytest.mark.parametrize("accumulate", [False, True])
def test_gemm_split_k(name, m, n, k, accumulate):
    """Few output tiles: the GEMM cuts K into parts (partial planes in the workspace, then one ordered
    reduction with the bias and the residual add).  Against the oracle, bit-identical on a second run,
    and within summation-order distance of the unsplit GEMM."""
    raw, w = wref(name, n, k, 111)
    rng = np.random.default_rng(112)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(113)).to(torch.bfloat16)
    b = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda()
    h0 = rng.standard_normal((m, n)).astype(np.float32) if accumulate else np.zeros((m, n), np.float32)
    W = GGUFTensor(raw, name, (n, k))
    ys = [_gemm(W, x.cuda(), y=torch.from_numpy(h0.copy()).cuda(), accumulate=accumulate, bias=b, split=True)
          for _ in range(2)]
    assert torch.equal(ys[0], ys[1])
    y1 = _gemm(W, x.cuda(), y=torch.from_numpy(h0.copy()).cuda(), accumulate=accumulate, bias=b)
    ref = h0 + x.float().numpy() @ w.T + b.cpu().numpy()
    tol = 1e-5 * max(1.0, k / 4096)
    assert rel_err(ys[0].cpu().numpy(), ref) < tol, rel_err(ys[0].cpu().numpy(), ref)
    assert rel_err(ys[0].cpu().numpy(), y1.cpu().numpy()) < tol


@pytest.mark.parametrize("m,n,k,accumulate", [(40, 300, 1792, False), (512, 4096, 7168, True), (96, 512, 3584, False)])
def test_gemm_pitched_rows(m, n, k, accumulate):
    """xm_qgemm_ex_pitched: Q6_K K-slices whose rows are not whole 16-byte units (the tensor-parallel down
    projection's slices: 1792 / 7168 / 3584 columns = 1470 / 5880 / 2940 bytes) padded to a 16-byte pitch."""
    raw, w = wref("Q6_K", n, k, 131)
    rb = len(raw) // n
    assert rb % 16
    pitch = (rb + 15) // 16 * 16
    pad = torch.zeros(n, pitch, dtype=torch.uint8)
    pad[:, :rb] = torch.from_numpy(np.frombuffer(raw, dtype=np.uint8).reshape(n, rb).copy())
    pad = pad.cuda()
    rng = np.random.default_rng(132)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(133)).to(torch.bfloat16)
    b = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda()
    h0 = rng.standard_normal((m, n)).astype(np.float32) if accumulate else np.zeros((m, n), np.float32)
    y = torch.from_numpy(h0.copy()).cuda()
    xd = x.cuda()
    ws = torch.empty(_lib.lib.xm_qgemm_workspace_size_n(m, n, k), dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib.xm_qgemm_ex_pitched(14, pad.data_ptr(), pitch, pad.numel(), n, k, xd.data_ptr(),
                                            _lib.DT_BF16, m, k, _lib.PRO_NONE, None, 1e-5, b.data_ptr(), y.data_ptr(),
                                            1 if accumulate else 0, ws.data_ptr(), ws.numel(), st), "pitched")
    torch.cuda.synchronize()
    ref = h0 + x.float().numpy() @ w.T + b.cpu().numpy()
    assert rel_err(y.cpu().numpy(), ref) < 1e-5 * max(1.0, k / 4096), rel_err(y.cpu().numpy(), ref)
    for bad in (rb, pitch - 16, pitch + 8):          # not a multiple of 16, or shorter than a row
        assert _lib.lib.xm_qgemm_ex_pitched(14, pad.data_ptr(), bad, pad.numel(), n, k, xd.data_ptr(), _lib.DT_BF16,
                                            m, k, _lib.PRO_NONE, None, 1e-5, None, y.data_ptr(), 0, ws.data_ptr(),
                                            ws.numel(), st) == _lib.XM_ERR_INVALID
