"""GPU linear operators over resident GGUF weights.

Mirrors the reference's ``LinearOp`` / ``FusedRMSNormLinearOp`` (ops.py:55-67,
ops.py:107-123): ``LinearOp(weight, bias).forward(x)`` returns
``fp32(x) @ W.T (+ bias)``.  ``weight`` is either a :class:`GGUFTensor` -- the
GGUF block bytes kept resident in HBM, multiplied by the fused dequant-GEMV
(m <= 8 rows) or the tensor-core dequant-GEMM (more rows) without ever
materialising the dequantized matrix -- or, as in the reference, a dense float
matrix (held on the GPU in fp32 and multiplied with a plain fp32 library GEMM).

``forward`` accepts a numpy array (returns numpy fp32, as the reference does), a
host torch tensor (returns a host tensor) or a CUDA tensor (returns a CUDA fp32
tensor).  Host inputs go through per-operator pinned staging buffers; after the
result is back on the host the device error word is checked, so a kernel whose
bounded wait gave up raises instead of returning wrong values.
"""

from __future__ import annotations

import numpy as np
import torch

from . import qtypes
from ._lib import DT_BF16, DT_F16, DT_F32, PRO_NONE, PRO_RMSNORM, PRO_SWIGLU, XMError, check, lib
from .gguf_dequant import dequantize_device

__all__ = ["GGUFTensor", "LinearOp", "FusedRMSNormLinearOp", "qlinear", "gemm_supported"]

_DT = {torch.float32: DT_F32, torch.bfloat16: DT_BF16, torch.float16: DT_F16}
# block types whose decode GEMV takes the fused prologues (integer-dot path)
_PROLOGUE_GEMV_TYPES = {"Q4_K", "Q5_K", "Q6_K", "Q8_0"}


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


def gemm_supported(qt: qtypes.QType, k: int) -> bool:
    """Whether the tensor-core GEMM takes rows of k weights of this type: k a
    multiple of 256 and a row a whole number of 16-byte units (its tensor map's
    row pitch)."""
    return k >= 256 and k % 256 == 0 and qtypes.row_bytes(qt, k) % 16 == 0


# Scratch buffers keyed by (device, stream): every call launches on the
# caller's current stream, so a buffer is only ever used by one stream and the
# caching allocator's stream-ordered reuse makes replacing it safe.
_WS: dict = {}


def _workspace(device, stream, nbytes: int) -> torch.Tensor:
    key = (device.index, stream.cuda_stream)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        with torch.cuda.stream(stream):
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _qmatmul(weight: GGUFTensor, x2: torch.Tensor, y: torch.Tensor, b, prologue: int, nw, eps: float,
             exact: bool, stream) -> None:
    """y[m][n] = pro(x2)[m] @ W.T (+ b); x2 is [m, kin] contiguous on the weight's device."""
    n, k = weight.shape
    m = x2.shape[0]
    kin = x2.shape[1]
    qt = weight.qtype
    dev = x2.device
    st = stream.cuda_stream
    dt = _DT[x2.dtype]
    if exact:
        if prologue != PRO_NONE:
            raise ValueError("the exact path takes no prologue")
        for m0 in range(0, m, 8):
            mm = min(8, m - m0)
            check(lib.xm_qgemv_exact(qt.type_id, weight.data.data_ptr(), weight.nbytes, n, k, x2[m0].data_ptr(), dt,
                                     mm, _ptr(b), y[m0].data_ptr(), st), "qgemv_exact")
        return
    gemm = gemm_supported(qt, k)
    if (m > 8 and gemm) or (m <= 8 and prologue != PRO_NONE and qt.name not in _PROLOGUE_GEMV_TYPES and gemm):
        ws = _workspace(dev, stream, lib.xm_qgemm_workspace_size_n(m, n, k))
        check(lib.xm_qgemm_ex(qt.type_id, weight.data.data_ptr(), weight.nbytes, n, k, x2.data_ptr(), dt, m, kin,
                              prologue, _ptr(nw), eps, _ptr(b), y.data_ptr(), 0, ws.data_ptr(), ws.numel(), st),
              "qgemm")
        return
    if prologue != PRO_NONE and qt.name not in _PROLOGUE_GEMV_TYPES:
        if prologue == PRO_SWIGLU:
            raise NotImplementedError(f"SwiGLU prologue for {qt.name} rows of {k} (no fused path at this shape)")
        xn = torch.empty((m, k), dtype=torch.float32, device=dev)
        check(lib.xm_rmsnorm(x2.data_ptr(), dt, m, k, kin, _ptr(nw), eps, xn.data_ptr(), st), "rmsnorm")
        x2, kin, dt, prologue = xn, k, DT_F32, PRO_NONE
    wsz = lib.xm_qgemv_workspace_size(k, min(8, m))
    ws = _workspace(dev, stream, max(wsz, 16))
    for m0 in range(0, m, 8):
        mm = min(8, m - m0)
        if prologue == PRO_NONE:
            st_ = lib.xm_qgemv(qt.type_id, weight.data.data_ptr(), weight.nbytes, n, k, x2[m0].data_ptr(), dt, mm,
                               _ptr(b), y[m0].data_ptr(), ws.data_ptr(), ws.numel(), st)
        else:
            st_ = lib.xm_qgemv_ex(qt.type_id, weight.data.data_ptr(), weight.nbytes, n, k, x2[m0].data_ptr(), dt, mm,
                                  kin, prologue, _ptr(nw), eps, _ptr(b), y[m0].data_ptr(), 0, ws.data_ptr(),
                                  ws.numel(), st)
        check(st_, "qgemv")


def qlinear(weight: GGUFTensor, x: torch.Tensor, bias: torch.Tensor | None = None, exact: bool = False,
            prologue: int = PRO_NONE, norm_weight: torch.Tensor | None = None, eps: float = 1e-5,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """y = pro(x) @ dequant(W).T (+ bias) on the GPU, fp32 out; x is a CUDA [..., k] tensor
    ([..., 2k] for the SwiGLU prologue).  ``out`` (fp32 [m, n], contiguous) receives the result if given."""
    n, k = weight.shape
    kin = 2 * k if prologue == PRO_SWIGLU else k
    if x.shape[-1] != kin:
        raise ValueError(f"x has {x.shape[-1]} features, weight expects {kin}")
    lead = x.shape[:-1]
    m = int(np.prod(lead)) if len(lead) else 1
    if x.dtype not in _DT:
        x = x.float()
    x2 = x.reshape(m, kin).contiguous()
    y = out if out is not None else torch.empty((m, n), dtype=torch.float32, device=x.device)
    b = None if bias is None else bias.to(device=x.device, dtype=torch.float32).contiguous()
    nw = None if norm_weight is None else norm_weight.to(device=x.device, dtype=torch.float32).contiguous()
    if m == 0:
        return y.reshape(*lead, n)
    with torch.cuda.device(x.device):
        _qmatmul(weight, x2, y, b, prologue, nw, eps, exact, torch.cuda.current_stream(x.device))
    return y.reshape(*lead, n)


class _HostIO:
    """Pinned staging buffers of one operator for host inputs: the activation
    goes host -> pinned -> device, the result device -> pinned -> host, and the
    device error word is copied behind the result on the same stream, so one
    stream synchronisation covers the whole call."""

    def __init__(self):
        self.key = None
        self.status = torch.zeros(1, dtype=torch.int32).pin_memory()

    def get(self, m, kin, n, dtype, device):
        key = (m, kin, n, dtype, device)
        if key != self.key:
            self.pin_in = torch.empty((m, kin), dtype=dtype).pin_memory()
            self.dev_in = torch.empty((m, kin), dtype=dtype, device=device)
            self.dev_out = torch.empty((m, n), dtype=torch.float32, device=device)
            self.pin_out = torch.empty((m, n), dtype=torch.float32).pin_memory()
            self.key = key
        return self


def _run_host(op, x, kin, n, fn):
    """Host-input path shared by the operators: x (numpy or host tensor) -> fn(dev_in, dev_out) -> host."""
    dev = op.device
    numpy_in = not isinstance(x, torch.Tensor)
    if numpy_in:
        xa = np.asarray(x, dtype=np.float32)
        xt = torch.from_numpy(np.ascontiguousarray(xa))
    else:
        xt = x if x.dtype in _DT else x.float()
    lead = tuple(xt.shape[:-1])
    if xt.shape[-1] != kin:
        raise ValueError(f"x has {xt.shape[-1]} features, expected {kin}")
    m = int(np.prod(lead)) if lead else 1
    io = op._io.get(m, kin, n, xt.dtype, dev)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        io.pin_in.copy_(xt.reshape(m, kin))
        io.dev_in.copy_(io.pin_in, non_blocking=True)
        if m:
            fn(io.dev_in, io.dev_out)
        io.pin_out.copy_(io.dev_out, non_blocking=True)
        check(lib.xm_device_status_async(io.status.data_ptr(), stream.cuda_stream), "device status")
        stream.synchronize()
        if int(io.status[0]):
            lib.xm_device_status(1)
            raise XMError(f"{type(op).__name__}: a bounded wait inside a kernel gave up (device error word "
                          f"{int(io.status[0])}); the result is not valid")
    res = io.pin_out.reshape(*lead, n)
    return res.numpy().copy() if numpy_in else res.clone()


def _dense_weight(weight):
    w = weight if isinstance(weight, torch.Tensor) else torch.from_numpy(np.asarray(weight, dtype=np.float32))
    if w.ndim != 2:
        raise ValueError(f"LinearOp weight must be 2-D, got shape {tuple(w.shape)}")
    dev = w.device if w.is_cuda else torch.device("cuda", torch.cuda.current_device())
    return w.to(device=dev, dtype=torch.float32).contiguous()


class LinearOp:
    """``out = x @ W.T (+ bias)`` (ops.py:55-67).

    ``weight``: a :class:`GGUFTensor` (quantized blocks resident on the GPU) or
    a dense float matrix [n, k] as the reference takes (numpy or torch)."""

    op_type = "linear"

    def __init__(self, weight, bias=None):
        if isinstance(weight, GGUFTensor):
            self.weight = weight
            self.dense = None
        else:
            self.dense = _dense_weight(weight)
            self.weight = None
        dev = self.device
        self.bias = None
        if bias is not None:
            self.bias = torch.as_tensor(np.asarray(bias, dtype=np.float32) if not isinstance(bias, torch.Tensor)
                                        else bias, dtype=torch.float32).to(dev).contiguous()
        self._io = _HostIO()

    @property
    def device(self):
        return self.weight.device if self.weight is not None else self.dense.device

    @property
    def out_features(self):
        return self.weight.shape[0] if self.weight is not None else self.dense.shape[0]

    @property
    def in_features(self):
        return self.weight.shape[1] if self.weight is not None else self.dense.shape[1]

    def _device_forward(self, x2, y):
        if self.weight is not None:
            qlinear(self.weight, x2, self.bias, out=y)
        elif self.bias is not None:
            torch.addmm(self.bias, x2.float(), self.dense.T, out=y)
        else:
            torch.mm(x2.float(), self.dense.T, out=y)

    def forward(self, x):
        n, k = self.out_features, self.in_features
        if isinstance(x, torch.Tensor) and x.is_cuda:
            lead = x.shape[:-1]
            if x.shape[-1] != k:
                raise ValueError(f"x has {x.shape[-1]} features, weight expects {k}")
            m = int(np.prod(lead)) if len(lead) else 1
            x2 = (x if x.dtype in _DT else x.float()).reshape(m, k).contiguous()
            y = torch.empty((m, n), dtype=torch.float32, device=x.device)
            if m:
                with torch.cuda.device(x.device):
                    self._device_forward(x2, y)
            return y.reshape(*lead, n)
        return _run_host(self, x, k, n, self._device_forward)

    __call__ = forward

    def __repr__(self):
        return f"<{self.__class__.__name__} op_type={self.op_type}>"


class FusedRMSNormLinearOp:
    """``rms_norm(x) * norm_weight`` then ``@ W.T (+ bias)`` (ops.py:107-123).

    For a :class:`GGUFTensor` the norm runs inside the matmul's activation
    prologue (decode GEMV for m <= 8 rows of Q4_K/Q5_K/Q6_K/Q8_0, the
    tensor-core GEMM's activation preparation otherwise); for a dense weight
    it is a separate kernel ahead of the fp32 library GEMM."""

    op_type = "fused_rmsnorm_linear"

    def __init__(self, norm_weight, linear_weight, linear_bias=None, eps=1e-5):
        self.linear = LinearOp(linear_weight, linear_bias)
        self.norm_weight = torch.as_tensor(np.asarray(norm_weight, dtype=np.float32)).to(self.linear.device)
        self.eps = float(eps)
        self._io = _HostIO()

    @property
    def device(self):
        return self.linear.device

    def _device_forward(self, x2, y):
        lin = self.linear
        if lin.weight is not None:
            qlinear(lin.weight, x2, lin.bias, prologue=PRO_RMSNORM, norm_weight=self.norm_weight, eps=self.eps,
                    out=y)
            return
        m, k = x2.shape
        xn = torch.empty((m, k), dtype=torch.float32, device=x2.device)
        check(lib.xm_rmsnorm(x2.data_ptr(), _DT[x2.dtype], m, k, k, self.norm_weight.data_ptr(), self.eps,
                             xn.data_ptr(), torch.cuda.current_stream(x2.device).cuda_stream), "rmsnorm")
        lin._device_forward(xn, y)

    def forward(self, x):
        n, k = self.linear.out_features, self.linear.in_features
        if isinstance(x, torch.Tensor) and x.is_cuda:
            lead = x.shape[:-1]
            if x.shape[-1] != k:
                raise ValueError(f"x has {x.shape[-1]} features, weight expects {k}")
            m = int(np.prod(lead)) if len(lead) else 1
            x2 = (x if x.dtype in _DT else x.float()).reshape(m, k).contiguous()
            y = torch.empty((m, n), dtype=torch.float32, device=x.device)
            if m:
                with torch.cuda.device(x.device):
                    self._device_forward(x2, y)
            return y.reshape(*lead, n)
        return _run_host(self, x, k, n, self._device_forward)

    __call__ = forward

    def __repr__(self):
        return f"<{self.__class__.__name__} op_type={self.op_type}>"

