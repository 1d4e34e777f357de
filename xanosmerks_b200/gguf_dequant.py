"""GPU drop-in for the reference's GGUF dequantization entry points.

Mirrors gguf_dequant.py of the reference: ``dequantize(raw_bytes, tensor_type,
shape)`` (gguf_dequant.py:477-523), the per-type ``dequant_<q>(raw_bytes,
shape)`` functions (gguf_dequant.py:25-455) and ``DEQUANT_FUNCS``
(gguf_dequant.py:461-474), with the same type-name folding, the same fp16
result (bit for bit) and the same exceptions (``NotImplementedError`` for
IQ*/TQ*/unknown types, ``ValueError`` for sizes that do not fit).

Inputs may be host bytes (``bytes``/``bytearray``/``memoryview``/numpy array):
the blocks are copied to the GPU, unpacked there and the result comes back as
a numpy ``float16`` array, exactly what the reference returns.  A CUDA
``torch.uint8`` tensor stays on the device and the result is a CUDA tensor
(``float16``, or ``float32`` with ``out_dtype="float32"`` for the value before
the fp16 cast).
"""

from __future__ import annotations

from functools import partial

import numpy as np
import torch

from . import qtypes
from ._lib import DT_F16, DT_F32, check, lib

__all__ = [
    "dequant_q4_0", "dequant_q4_1", "dequant_q5_0", "dequant_q5_1",
    "dequant_q8_0", "dequant_q8_1",
    "dequant_q2_k", "dequant_q3_k",
    "dequant_q4_k", "dequant_q5_k", "dequant_q6_k", "dequant_q8_k",
    "DEQUANT_FUNCS", "dequantize", "dequantize_device",
]


def _shape_tuple(shape):
    if isinstance(shape, (int, np.integer)):
        return (int(shape),)
    return tuple(int(s) for s in shape)


def _stream_handle(device):
    return torch.cuda.current_stream(device).cuda_stream


def dequantize_device(raw: torch.Tensor, qt: qtypes.QType, n_elements: int, out_dtype=torch.float16) -> torch.Tensor:
    """Unpack ``n_elements`` of type ``qt`` from a CUDA uint8 tensor; returns a flat CUDA tensor."""
    if not raw.is_cuda:
        raise ValueError("dequantize_device expects a CUDA tensor")
    raw = raw.contiguous()
    out = torch.empty(n_elements, dtype=out_dtype, device=raw.device)
    dt = DT_F16 if out_dtype == torch.float16 else DT_F32
    if out_dtype not in (torch.float16, torch.float32):
        raise ValueError("out_dtype must be float16 or float32")
    if not qt.quantized and raw.numel() != n_elements * qt.record:
        # the reference reads plain types with np.frombuffer(...).reshape(shape)
        raise ValueError(f"{qt.name}: buffer of {raw.numel()} bytes does not hold exactly {n_elements} elements")
    with torch.cuda.device(raw.device):
        check(lib.xm_dequantize(qt.type_id, raw.data_ptr(), raw.numel(), n_elements, out.data_ptr(), dt,
                                _stream_handle(raw.device)), f"dequantize {qt.name}")
    return out


def _host_bytes(raw_bytes) -> np.ndarray:
    if isinstance(raw_bytes, np.ndarray):
        return np.ascontiguousarray(raw_bytes).view(np.uint8).reshape(-1)
    return np.frombuffer(raw_bytes, dtype=np.uint8)


def _dequantize(raw_bytes, qt: qtypes.QType, shape, out_dtype="float16", device=None):
    shape = _shape_tuple(shape)
    n = int(np.prod(shape)) if len(shape) else 1
    odt = torch.float16 if out_dtype in ("float16", np.float16, torch.float16) else torch.float32
    if isinstance(raw_bytes, torch.Tensor) and raw_bytes.is_cuda:
        return dequantize_device(raw_bytes.view(torch.uint8).reshape(-1), qt, n, odt).reshape(shape)
    host = _host_bytes(raw_bytes)
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    d_raw = torch.from_numpy(host.copy()).to(dev, non_blocking=False) if host.size else torch.empty(0, dtype=torch.uint8, device=dev)
    out = dequantize_device(d_raw, qt, n, odt)
    res = out.cpu().numpy().reshape(shape)
    return res


def dequantize(raw_bytes, tensor_type, shape, out_dtype="float16", device=None):
    """Dequantize a GGUF tensor on the GPU; same contract as the reference ``dequantize``.

    ``raw_bytes``: host buffer (returns numpy) or CUDA uint8 tensor (returns a
    CUDA tensor).  ``tensor_type``: GGUF type name (``Q4_K_M`` folds to
    ``Q4_K``; IQ*/TQ* raise ``NotImplementedError``).  ``shape``: output shape
    (flat GGUF element order).
    """
    qt = qtypes.normalize(tensor_type)
    return _dequantize(raw_bytes, qt, shape, out_dtype, device)


def _per_type(name, raw_bytes, shape, out_dtype="float16", device=None):
    return _dequantize(raw_bytes, qtypes.BY_NAME[name], shape, out_dtype, device)


dequant_q4_0 = partial(_per_type, "Q4_0")
dequant_q4_1 = partial(_per_type, "Q4_1")
dequant_q5_0 = partial(_per_type, "Q5_0")
dequant_q5_1 = partial(_per_type, "Q5_1")
dequant_q8_0 = partial(_per_type, "Q8_0")
dequant_q8_1 = partial(_per_type, "Q8_1")
dequant_q2_k = partial(_per_type, "Q2_K")
dequant_q3_k = partial(_per_type, "Q3_K")
dequant_q4_k = partial(_per_type, "Q4_K")
dequant_q5_k = partial(_per_type, "Q5_K")
dequant_q6_k = partial(_per_type, "Q6_K")
dequant_q8_k = partial(_per_type, "Q8_K")

DEQUANT_FUNCS = {
    "Q4_0": dequant_q4_0, "Q4_1": dequant_q4_1, "Q5_0": dequant_q5_0, "Q5_1": dequant_q5_1,
    "Q8_0": dequant_q8_0, "Q8_1": dequant_q8_1, "Q2_K": dequant_q2_k, "Q3_K": dequant_q3_k,
    "Q4_K": dequant_q4_k, "Q5_K": dequant_q5_k, "Q6_K": dequant_q6_k, "Q8_K": dequant_q8_k,
}
