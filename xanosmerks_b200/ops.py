"""GPU linear operators over resident GGUF weights.

Mirrors the reference's ``LinearOp`` / ``FusedRMSNormLinearOp`` (ops.py:55-67,
ops.py:107-123): ``LinearOp(weight, bias).forward(x)`` returns
``fp32(x) @ W.T (+ bias)``.  Here ``weight`` is a :class:`GGUFTensor` -- the
GGUF block bytes kept resident in HBM -- and the product runs in the fused
dequant-GEMV/GEMM kernels, so the dequantized matrix is never materialised.

``forward`` accepts a numpy array (returns numpy fp32, as the reference does)
or a CUDA tensor (returns a CUDA fp32 tensor).
"""

from __future__ import annotations

import numpy as np
import torch

from . import qtypes
from ._lib import DT_BF16, DT_F16, DT_F32, check, lib
from .gguf_dequant import dequantize_device

__all__ = ["GGUFTensor", "LinearOp", "FusedRMSNormLinearOp", "qlinear"]

_DT = {torch.float32: DT_F32, torch.bfloat16: DT_BF16, torch.float16: DT_F16}
# block types with a tensor-core GEMM for m > 8 (others use the GEMV on groups of 8 rows)
_TC_TYPES = {"Q4_K"}


class GGUFTensor:
    """A 2-D quantized weight W[n][k] held on the GPU as raw GGUF block bytes.

    ``shape`` is the HF layout (n rows, k columns); the GGUF file stores the
    same bytes with dims ``[k, n]`` (readers.py:801-828).
    """

    def __init__(self, raw, tensor_type: str, shape, device=None):
        self.qtype = qtypes.normalize(tensor_type)
        if not self.qtype.quantized:
            raise NotImplementedError(f"GGUFTensor holds block-quantized types, not {self.qtype.name}")
        n, k = (int(s) for s in shape)
        self.shape = (n, k)
        need = qtypes.row_bytes(self.qtype, k) * n
        if isinstance(raw, torch.Tensor):
            data = raw.view(torch.uint8).reshape(-1)
            if device is not None:
                data = data.to(device)
        else:
            host = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray)
                                        else raw.view(np.uint8).reshape(-1))
            dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
            data = torch.from_numpy(host.copy()).to(dev)
        if data.numel() < need:
            raise ValueError(f"{self.qtype.name} {shape}: need {need} bytes, got {data.numel()}")
        if not data.is_cuda:
            raise ValueError("GGUFTensor data must live on a CUDA device")
        self.data = data[:need].contiguous()

    @property
    def nbytes(self) -> int:
        return self.data.numel()

    @property
    def device(self):
        return self.data.device

    def dequantize(self, out_dtype=torch.float16) -> torch.Tensor:
        """Reference-exact fp16 (or pre-cast fp32) matrix, shape (n, k)."""
        return dequantize_device(self.data, self.qtype, self.shape[0] * self.shape[1], out_dtype).view(self.shape)

    def __repr__(self):
        return f"<GGUFTensor {self.qtype.name} {self.shape} on {self.device}>"


_WS: dict = {}


def _workspace(device, nbytes: int) -> torch.Tensor:
    key = (device.type, device.index)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def qlinear(weight: GGUFTensor, x: torch.Tensor, bias: torch.Tensor | None = None, exact: bool = False) -> torch.Tensor:
    """y = x @ dequant(W).T (+ bias) on the GPU, fp32 out; x is a CUDA [..., k] tensor."""
    n, k = weight.shape
    if x.shape[-1] != k:
        raise ValueError(f"x has {x.shape[-1]} features, weight expects {k}")
    lead = x.shape[:-1]
    m = int(np.prod(lead)) if len(lead) else 1
    if x.dtype not in _DT:
        x = x.float()
    x2 = x.reshape(m, k).contiguous()
    y = torch.empty((m, n), dtype=torch.float32, device=x.device)
    b = None
    if bias is not None:
        b = bias.to(device=x.device, dtype=torch.float32).contiguous()
    stream = torch.cuda.current_stream(x.device).cuda_stream
    with torch.cuda.device(x.device):
        if m > 8 and not exact and weight.qtype.name in _TC_TYPES:
            wsz = lib.xm_qgemm_workspace_size(m, k)
            ws = _workspace(x.device, wsz)
            check(lib.xm_qgemm(weight.qtype.type_id, weight.data.data_ptr(), weight.nbytes, n, k, x2.data_ptr(),
                               _DT[x2.dtype], m, b.data_ptr() if b is not None else None, y.data_ptr(),
                               ws.data_ptr(), ws.numel(), stream), "qgemm")
            return y.reshape(*lead, n)
        for m0 in range(0, m, 8):
            mm = min(8, m - m0)
            xs = x2[m0:m0 + mm]
            ys = y[m0:m0 + mm]
            if exact:
                st = lib.xm_qgemv_exact(weight.qtype.type_id, weight.data.data_ptr(), weight.nbytes, n, k,
                                        xs.data_ptr(), _DT[x2.dtype], mm, b.data_ptr() if b is not None else None,
                                        ys.data_ptr(), stream)
            else:
                wsz = lib.xm_qgemv_workspace_size(k, mm)
                ws = _workspace(x.device, wsz)
                st = lib.xm_qgemv(weight.qtype.type_id, weight.data.data_ptr(), weight.nbytes, n, k,
                                  xs.data_ptr(), _DT[x2.dtype], mm, b.data_ptr() if b is not None else None,
                                  ys.data_ptr(), ws.data_ptr(), ws.numel(), stream)
            check(st, "qgemv")
    return y.reshape(*lead, n)


def _to_device_x(x, device):
    """(device tensor, how to return): "numpy" for array input, "cpu" for a host
    torch tensor (copied with non_blocking when pinned), None for a CUDA tensor."""
    if isinstance(x, torch.Tensor):
        if x.is_cuda:
            return x, None
        return x.to(device, non_blocking=x.is_pinned()), "cpu"
    arr = np.asarray(x, dtype=np.float32)
    return torch.from_numpy(np.ascontiguousarray(arr)).to(device), "numpy"


def _back(y, how):
    if how == "numpy":
        return y.cpu().numpy()
    if how == "cpu":
        return y.cpu()
    return y


class LinearOp:
    """``out = x @ W.T (+ bias)`` with W resident as GGUF blocks (ops.py:55-67)."""

    op_type = "linear"

    def __init__(self, weight: GGUFTensor, bias=None):
        if not isinstance(weight, GGUFTensor):
            raise TypeError("LinearOp expects a GGUFTensor weight (quantized blocks resident on the GPU)")
        self.weight = weight
        self.bias = None
        if bias is not None:
            self.bias = torch.as_tensor(np.asarray(bias, dtype=np.float32) if not isinstance(bias, torch.Tensor)
                                        else bias, dtype=torch.float32).to(weight.device)

    def forward(self, x):
        xd, how = _to_device_x(x, self.weight.device)
        return _back(qlinear(self.weight, xd, self.bias), how)

    __call__ = forward

    def __repr__(self):
        return f"<{self.__class__.__name__} op_type={self.op_type}>"


class FusedRMSNormLinearOp:
    """``rms_norm(x) * norm_weight`` then ``@ W.T`` (ops.py:107-123)."""

    op_type = "fused_rmsnorm_linear"

    def __init__(self, norm_weight, linear_weight: GGUFTensor, linear_bias=None, eps=1e-5):
        self.linear = LinearOp(linear_weight, linear_bias)
        self.norm_weight = torch.as_tensor(np.asarray(norm_weight, dtype=np.float32)).to(linear_weight.device)
        self.eps = eps

    def forward(self, x):
        xd, how = _to_device_x(x, self.linear.weight.device)
        xf = xd.float()
        rms = torch.sqrt(torch.mean(xf * xf, dim=-1, keepdim=True) + self.eps)
        return _back(qlinear(self.linear.weight, (xf / rms) * self.norm_weight, self.linear.bias), how)

    __call__ = forward
