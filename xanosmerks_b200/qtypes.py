"""GGUF tensor-type table shared by the host API, the tests and the oracle.

Type ids are the GGML numbers the reference uses in its GGUF reader
(dtype_map.py:33-65, ``GGUF_TENSOR_TYPES``); block geometry follows
``GGUF_TYPE_BLOCK_SIZE`` (dtype_map.py:68-79).  The same ids are the ``qtype``
argument of every entry point in ``include/xm_gguf.h``.
"""

from __future__ import annotations

from dataclasses import dataclass

# GGML type ids (dtype_map.py:33-65).
F32 = 0
F16 = 1
Q4_0 = 2
Q4_1 = 3
Q5_0 = 6
Q5_1 = 7
Q8_0 = 8
Q8_1 = 9
Q2_K = 10
Q3_K = 11
Q4_K = 12
Q5_K = 13
Q6_K = 14
Q8_K = 15
I8 = 24
I16 = 25
I32 = 26
I64 = 27
BF16 = 30


@dataclass(frozen=True)
class QType:
    name: str
    type_id: int
    qk: int          # elements per block (1 for plain types)
    record: int      # bytes per block
    quantized: bool


_TABLE = [
    QType("F32", F32, 1, 4, False),
    QType("F16", F16, 1, 2, False),
    QType("BF16", BF16, 1, 2, False),
    QType("I8", I8, 1, 1, False),
    QType("I16", I16, 1, 2, False),
    QType("I32", I32, 1, 4, False),
    QType("I64", I64, 1, 8, False),
    QType("Q4_0", Q4_0, 32, 18, True),
    QType("Q4_1", Q4_1, 32, 20, True),
    QType("Q5_0", Q5_0, 32, 22, True),
    QType("Q5_1", Q5_1, 32, 24, True),
    QType("Q8_0", Q8_0, 32, 34, True),
    QType("Q8_1", Q8_1, 32, 40, True),
    QType("Q2_K", Q2_K, 256, 84, True),
    QType("Q3_K", Q3_K, 256, 110, True),
    QType("Q4_K", Q4_K, 256, 144, True),
    QType("Q5_K", Q5_K, 256, 176, True),
    QType("Q6_K", Q6_K, 256, 210, True),
    QType("Q8_K", Q8_K, 256, 292, True),
]

BY_NAME = {q.name: q for q in _TABLE}
BY_ID = {q.type_id: q for q in _TABLE}

# The twelve block formats ``DEQUANT_FUNCS`` dispatches (gguf_dequant.py:461-474).
QUANT_NAMES = ["Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0", "Q8_1",
               "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_K"]

# Aliases accepted for the plain types (gguf_dequant.py:503-518).
_PLAIN_ALIASES = {
    "F16": "F16", "FP16": "F16",
    "F32": "F32", "FP32": "F32",
    "BF16": "BF16",
    "I8": "I8", "INT8": "I8",
    "I16": "I16", "INT16": "I16",
    "I32": "I32", "INT32": "I32",
    "I64": "I64", "INT64": "I64",
}

_K_PREFIXES = ("Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_K")


def normalize(tensor_type: str) -> QType:
    """Map a tensor-type string to its table entry, as the reference dispatcher does.

    Follows gguf_dequant.py:477-523: upper-case the name, fold ``Q4_K_M``-style
    suffixes onto the base K-quant by prefix, raise ``NotImplementedError`` for
    IQ*/TQ* and for any name that is not handled.
    """
    ttype = tensor_type.upper()
    for p in _K_PREFIXES:
        if ttype.startswith(p):
            return BY_NAME[p]
    if ttype.startswith("IQ"):
        raise NotImplementedError(
            f"{tensor_type} (IQ quantization) is not implemented; "
            f"use Q4_K_M or Q8_0 models.")
    if ttype.startswith("TQ"):
        raise NotImplementedError(
            f"{tensor_type} (ternary quantization) is not implemented.")
    if ttype in _PLAIN_ALIASES:
        return BY_NAME[_PLAIN_ALIASES[ttype]]
    if ttype in BY_NAME:
        return BY_NAME[ttype]
    raise NotImplementedError(f"Type {tensor_type} is not supported")


def row_bytes(qt: QType, k: int) -> int:
    """Bytes of one GGUF row of ``k`` elements (``k`` a multiple of the block)."""
    if k % qt.qk:
        raise ValueError(f"{qt.name}: row length {k} is not a multiple of {qt.qk}")
    return (k // qt.qk) * qt.record
