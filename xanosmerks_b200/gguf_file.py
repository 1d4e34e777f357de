"""GGUF container: parse the header and load the tensors onto the GPU.

Mirrors the reference's container side of the quantized-weight path:

* ``parse_gguf(path)`` returns the same dictionary as readers.py:769-856
  (version, counts, metadata, tensor infos with type name, offset, byte size
  and element count, alignment, data start and sizes) and raises the same
  kinds of error: ``CorruptedGGUFError`` for a bad magic, version, metadata
  type, array length or dimension count, or a metadata value that cannot be
  read; ``EOFError`` for a header cut short elsewhere.
* ``load_gguf(path)`` is loaders.py:302-385 for this library: instead of
  dequantizing every tensor to a host array at load (loaders.py:343), each
  2-D block-quantized weight stays quantized and resident on the GPU as a
  ``GGUFTensor`` (the form ``LinearOp``, ``MoELayer`` and ``LlamaDecoder``
  consume), and every other tensor is unpacked on the GPU by the dequant
  kernel.  ``keep_quantized=False`` unpacks everything, like the reference.

The header is read with ``struct.unpack_from`` over a memory map; arrays of
scalars in the metadata are read in one ``numpy.frombuffer`` each.
"""

from __future__ import annotations

import mmap
import struct
from pathlib import Path

import numpy as np
import torch

from . import qtypes

__all__ = ["CorruptedGGUFError", "UnsupportedDTypeError", "WeightLoadError", "GGUF_TENSOR_TYPES",
           "gguf_tensor_size_in_bytes", "parse_gguf", "load_gguf"]


class CorruptedGGUFError(ValueError):
    """The file is not a well-formed GGUF container."""


class UnsupportedDTypeError(NotImplementedError):
    """A tensor's block type has no unpacker (IQ*/TQ* and unknown types)."""


class WeightLoadError(RuntimeError):
    """A tensor could not be read or unpacked."""


# Tensor type ids of the GGUF format with (name, elements per block, bytes per
# block); the same numbering and sizes as dtype_map.py:33-80.
_FORMAT = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20),
    6: ("Q5_0", 32, 22), 7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34), 9: ("Q8_1", 32, 40),
    10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176),
    14: ("Q6_K", 256, 210), 15: ("Q8_K", 256, 292), 16: ("IQ2_XXS", 256, 66), 17: ("IQ2_XS", 256, 74),
    18: ("IQ3_XXS", 256, 98), 19: ("IQ1_S", 256, 50), 20: ("IQ4_NL", 32, 18), 21: ("IQ3_S", 256, 110),
    22: ("IQ2_S", 256, 82), 23: ("IQ4_XS", 256, 136), 24: ("I8", 1, 1), 25: ("I16", 1, 2),
    26: ("I32", 1, 4), 27: ("I64", 1, 8), 28: ("F64", 1, 8), 29: ("IQ1_M", 256, 56),
    30: ("BF16", 1, 2), 34: ("TQ1_0", 256, 54), 35: ("TQ2_0", 256, 66),
}
GGUF_TENSOR_TYPES = {i: v[0] for i, v in _FORMAT.items()}
_BLOCK = {v[0]: (v[1], v[2]) for v in _FORMAT.values()}


def gguf_type_name(type_id: int) -> str:
    return GGUF_TENSOR_TYPES.get(type_id, f"UNKNOWN_{type_id}")


def gguf_tensor_size_in_bytes(type_id: int, num_elements: int) -> int:
    """Bytes of `num_elements` of a type: whole blocks, the last one partly used."""
    name = gguf_type_name(type_id)
    if name not in _BLOCK:
        raise ValueError(f"unknown GGUF tensor type: {name}")
    qk, rec = _BLOCK[name]
    return (num_elements + qk - 1) // qk * rec


# metadata value types: id -> (name, struct format, numpy dtype for arrays)
_META = {
    0: ("uint8", "<B", "<u1"), 1: ("int8", "<b", "<i1"), 2: ("uint16", "<H", "<u2"), 3: ("int16", "<h", "<i2"),
    4: ("uint32", "<I", "<u4"), 5: ("int32", "<i", "<i4"), 6: ("float32", "<f", "<f4"), 7: ("bool", "<B", "<u1"),
    8: ("string", None, None), 9: ("array", None, None), 10: ("uint64", "<Q", "<u8"), 11: ("int64", "<q", "<i8"),
    12: ("float64", "<d", "<f8"),
}
_MAX_ARRAY = 10_000_000


class _Cursor:
    """Little-endian reads from a buffer; running out of bytes is EOFError."""

    def __init__(self, buf, name):
        self.buf, self.pos, self.name = buf, 0, name

    def take(self, n):
        if self.pos + n > len(self.buf):
            raise EOFError(f"expected {n} bytes at offset {self.pos}, the file ({self.name}) ends at {len(self.buf)}")
        p = self.pos
        self.pos += n
        return p

    def unpack(self, fmt, size):
        return struct.unpack_from(fmt, self.buf, self.take(size))[0]

    def u32(self):
        return self.unpack("<I", 4)

    def u64(self):
        return self.unpack("<Q", 8)

    def string(self):
        n = self.u64()
        p = self.take(n)
        return bytes(self.buf[p:p + n]).decode("utf-8", errors="replace")


def _meta_value(c: _Cursor, type_id: int):
    if type_id not in _META:
        raise CorruptedGGUFError(f"unknown metadata value type {type_id}")
    name, fmt, npdt = _META[type_id]
    if name == "string":
        return c.string()
    if name == "array":
        inner = c.u32()
        count = c.u64()
        if count > _MAX_ARRAY:
            raise CorruptedGGUFError(f"implausible array length {count}")
        if inner in _META and _META[inner][2] is not None:      # array of scalars: one read
            width = struct.calcsize(_META[inner][1])
            p = c.take(count * width)
            vals = np.frombuffer(c.buf, dtype=_META[inner][2], count=count, offset=p)
            if _META[inner][0] == "bool":
                return [bool(v) for v in vals.tolist()]
            return vals.tolist()
        return [_meta_value(c, inner) for _ in range(count)]
    v = c.unpack(fmt, struct.calcsize(fmt))
    return bool(v) if name == "bool" else v


def _human_size(num_bytes: float) -> str:
    for unit in ("B", "KB", "MB", "GB", "TB"):
        if num_bytes < 1024:
            return f"{num_bytes:.2f} {unit}"
        num_bytes /= 1024
    return f"{num_bytes:.2f} PB"


def _parse(buf, path: Path) -> dict:
    c = _Cursor(buf, path.name)
    p = c.take(4)
    if bytes(buf[p:p + 4]) != b"GGUF":
        raise CorruptedGGUFError(f"{path.name} is not a GGUF file")
    version = c.u32()
    if version < 1 or version > 5:
        raise CorruptedGGUFError(f"unsupported GGUF version {version}")
    tensor_count = c.u64()
    metadata_count = c.u64()
    metadata = {}
    for _ in range(metadata_count):
        key = c.string()
        type_id = c.u32()
        try:
            metadata[key] = _meta_value(c, type_id)
        except Exception as e:  # noqa: BLE001  (any failure inside a value names the key, like the reference)
            tname = _META.get(type_id, ("?",))[0]
            raise CorruptedGGUFError(f"cannot read metadata '{key}' ({tname}): {e}") from e
    alignment = metadata.get("general.alignment", 32)
    tensors = []
    for _ in range(tensor_count):
        name = c.string()
        n_dims = c.u32()
        if n_dims > 8:
            raise CorruptedGGUFError(f"tensor '{name}' has {n_dims} dimensions")
        dims = [c.u64() for _ in range(n_dims)]
        type_id = c.u32()
        offset = c.u64()
        num_elements = 1
        for d in dims:
            num_elements *= d
        try:
            size_bytes = gguf_tensor_size_in_bytes(type_id, num_elements)
        except ValueError:
            size_bytes = 0
        tensors.append({"name": name, "shape": dims, "type": gguf_type_name(type_id), "type_id": type_id,
                        "offset": offset, "size_bytes": size_bytes, "num_elements": num_elements if dims else 0})
    data_start = (c.pos + alignment - 1) // alignment * alignment
    total = len(buf)
    return {"format": "gguf", "file": str(path), "version": version, "tensor_count": tensor_count,
            "metadata_count": metadata_count, "metadata": metadata, "tensors": tensors,
            "architecture": metadata.get("general.architecture", "unknown"),
            "model_name": metadata.get("general.name", ""), "alignment": alignment, "data_start": data_start,
            "data_size_bytes": total - data_start, "total_size_bytes": total,
            "total_size_human": _human_size(total)}


def parse_gguf(filepath) -> dict:
    """Parse a GGUF file's header (readers.py:769-856); tensor data is not read."""
    path = Path(filepath)
    if not path.exists():
        raise CorruptedGGUFError(f"file not found: {filepath}")
    with open(path, "rb") as f:
        if path.stat().st_size == 0:
            return _parse(b"", path)
        with mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as mm:
            return _parse(mm, path)


def load_gguf(path, dtype="float16", device=None, keep_quantized=True):
    """Load every tensor of a GGUF file onto the GPU (loaders.py:302-385).

    Returns ``(tensors, meta)``.  With ``keep_quantized`` (default) a 2-D
    block-quantized tensor whose rows hold whole blocks becomes a resident
    ``GGUFTensor`` of HF shape ``(dims[1], dims[0])``; every other tensor is
    unpacked on the GPU to a CUDA tensor of the reference's shape (the GGUF
    dims, as loaders.py:343 passes them) and cast to ``dtype``.
    ``meta`` carries the reference's keys (format, file, sizes, tensor count,
    architecture, model name, version, metadata, source dtypes).
    """
    from .gguf_dequant import dequantize
    from .ops import GGUFTensor

    path = Path(path)
    if not path.exists():
        raise WeightLoadError(f"file not found: {path}")
    try:
        info = parse_gguf(path)
    except Exception as e:  # noqa: BLE001
        raise WeightLoadError(f"cannot parse GGUF {path.name}: {e}") from e
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    target = getattr(torch, str(np.dtype(dtype)))
    file_size = path.stat().st_size
    tensors, source_dtypes = {}, {}
    with open(path, "rb") as f, mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as mm:
        for t in info["tensors"]:
            name, shape, tname = t["name"], [int(d) for d in t["shape"]], t["type"]
            start = info["data_start"] + t["offset"]
            end = start + t["size_bytes"]
            if end > file_size:
                raise WeightLoadError(f"tensor {name}: data runs past the end of the file")
            try:
                qt = qtypes.normalize(tname)
            except NotImplementedError as e:
                raise UnsupportedDTypeError(f"tensor {name}: type {tname} is not supported. {e}") from e
            host = np.frombuffer(mm, dtype=np.uint8, count=end - start, offset=start).copy()
            d_raw = torch.from_numpy(host).to(dev)
            try:
                if keep_quantized and qt.quantized and len(shape) == 2 and shape[0] % qt.qk == 0:
                    tensors[name] = GGUFTensor(d_raw, tname, (shape[1], shape[0]))
                    source_dtypes[name] = qt.name
                    continue
                arr = dequantize(d_raw, tname, shape)
            except NotImplementedError as e:
                raise UnsupportedDTypeError(f"tensor {name}: type {tname} is not supported. {e}") from e
            except Exception as e:  # noqa: BLE001
                raise WeightLoadError(f"cannot unpack {name} ({tname}): {e}") from e
            if arr.dtype != target:
                arr = arr.to(target)
            tensors[name] = arr
            source_dtypes[name] = str(arr.dtype).replace("torch.", "")
    meta = {"format": "gguf", "file": str(path), "file_size_bytes": file_size, "num_tensors": len(tensors),
            "architecture": info.get("architecture", "unknown"), "model_name": info.get("model_name", ""),
            "version": info.get("version"), "metadata": info.get("metadata", {}), "source_dtypes": source_dtypes}
    return tensors, meta
