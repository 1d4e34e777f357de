"""CPU oracle for GGUF block dequantization -- test infrastructure only.

This module is the checker for the CUDA dequant kernels.  It is imported only by
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``;
the product path (``xanosmerks_b200``) never imports it.

It restates, in vectorised numpy, the reference's per-qtype unpack
(gguf_dequant.py:17-523).  Each ``q_*`` function returns the float32 value the
reference holds *before* its final ``.astype(np.float16)``, reproducing the
reference's float32 operation order (separate multiply and add; no fused
multiply-add).  ``dequantize`` applies the same fp16 cast and the same type-name
normalisation and passthrough rules as the reference.

Parity of this restatement is pinned against the reference itself: the
fixtures under ``tests/golden/`` were produced by running the reference
functions (``tests/golden/make_golden.py``) and ``tests/test_oracle_golden.py``
checks this module against them bit for bit.
"""

from __future__ import annotations

import numpy as np

QK_SMALL = 32
QK_K = 256


def _blocks(raw, n_elements, qk, record):
    """(n_blocks, record) uint8 view, truncated as gguf_dequant.py:28-32 does."""
    if n_elements % qk:
        raise ValueError(f"{n_elements} elements is not a multiple of block size {qk}")
    n_blocks = n_elements // qk
    raw = np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw.view(np.uint8).reshape(-1)
    need = n_blocks * record
    if raw.size < need:
        raise ValueError(f"need {need} bytes for {n_blocks} blocks of {record} B, got {raw.size}")
    return raw[:need].reshape(n_blocks, record)


def _f16(b2):
    """Little-endian fp16 pairs -> float32, exact (gguf_dequant.py:17-19)."""
    return np.ascontiguousarray(b2).view(np.float16).reshape(-1).astype(np.float32)


def _f32(b4):
    return np.ascontiguousarray(b4).view(np.float32).reshape(-1)


def _interleave(lo, hi):
    """Element 2i = lo[i], 2i+1 = hi[i] (gguf_dequant.py:40-42)."""
    out = np.empty((lo.shape[0], lo.shape[1] * 2), dtype=lo.dtype)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    return out


def q4_0(raw, n):
    """gguf_dequant.py:25-45: fp16 d @0, 16 B nibbles @2; (v - 8) * d."""
    b = _blocks(raw, n, 32, 18)
    d = _f16(b[:, 0:2])
    qs = b[:, 2:18]
    v = _interleave(qs & 0x0F, qs >> 4).astype(np.float32)
    return ((v - np.float32(8.0)) * d[:, None]).reshape(-1)


def q4_1(raw, n):
    """gguf_dequant.py:51-72: d @0, m @2, nibbles @4; v * d + m."""
    b = _blocks(raw, n, 32, 20)
    d = _f16(b[:, 0:2])
    m = _f16(b[:, 2:4])
    qs = b[:, 4:20]
    v = _interleave(qs & 0x0F, qs >> 4).astype(np.float32)
    return (v * d[:, None] + m[:, None]).reshape(-1)


def _qh_bits(qh4):
    """Bit i of the little-endian u32 built from 4 bytes, i = 0..31 (gguf_dequant.py:94-95)."""
    u = np.ascontiguousarray(qh4).view(np.uint32).reshape(-1)
    return ((u[:, None] >> np.arange(32, dtype=np.uint32)) & 1).astype(np.int16)


def q5_0(raw, n):
    """gguf_dequant.py:78-105: d @0, qh u32 @2, nibbles @6.

    The 5th bit of element i is bit i of qh, applied after the interleave
    (gguf_dequant.py:97-102); then (v - 16) * d.
    """
    b = _blocks(raw, n, 32, 22)
    d = _f16(b[:, 0:2])
    qs = b[:, 6:22]
    v = _interleave(qs & 0x0F, qs >> 4).astype(np.int16)
    v = (v | (_qh_bits(b[:, 2:6]) << 4)) - 16
    return (v.astype(np.float32) * d[:, None]).reshape(-1)


def q5_1(raw, n):
    """gguf_dequant.py:111-137: d @0, m @2, qh @4, nibbles @8; v * d + m."""
    b = _blocks(raw, n, 32, 24)
    d = _f16(b[:, 0:2])
    m = _f16(b[:, 2:4])
    qs = b[:, 8:24]
    v = _interleave(qs & 0x0F, qs >> 4).astype(np.int16)
    v = v | (_qh_bits(b[:, 4:8]) << 4)
    return (v.astype(np.float32) * d[:, None] + m[:, None]).reshape(-1)


def q8_0(raw, n):
    """gguf_dequant.py:143-156: fp16 d @0, 32 x int8 @2; q * d."""
    b = _blocks(raw, n, 32, 34)
    d = _f16(b[:, 0:2])
    q = b[:, 2:34].view(np.int8).astype(np.float32)
    return (q * d[:, None]).reshape(-1)


def q8_1(raw, n):
    """gguf_dequant.py:162-176: fp32 d @0, fp32 m @4, 32 x int8 @8; (q * d) + m, two roundings."""
    b = _blocks(raw, n, 32, 40)
    d = _f32(b[:, 0:4])
    m = _f32(b[:, 4:8])
    q = b[:, 8:40].view(np.int8).astype(np.float32)
    return (q * d[:, None] + m[:, None]).reshape(-1)


def q2_k(raw, n):
    """gguf_dequant.py:183-223: scales[16] @0, qs[64] @16, d @80, dmin @82.

    For half h (128 outputs) and shift j: outputs 128h + 32j + l (l < 16) use
    scale byte 8h + 2j and qs[32h + l]; outputs 128h + 32j + 16 + l use scale
    byte 8h + 2j + 1 and qs[32h + 16 + l]; value (d*(sc&15))*((q >> 2j)&3) -
    dmin*(sc>>4).  The reference evaluates this in Python float64 and stores it
    into a float32 array; every product is exact there, so float64 followed by
    one cast to float32 reproduces it.
    """
    b = _blocks(raw, n, 256, 84)
    nb = b.shape[0]
    sc = b[:, 0:16].astype(np.int64)
    qs = b[:, 16:80].astype(np.int64)
    d = _f16(b[:, 80:82]).astype(np.float64)
    dmin = _f16(b[:, 82:84]).astype(np.float64)
    out = np.empty((nb, 256), dtype=np.float64)
    for h in range(2):
        for j in range(4):
            for part in range(2):
                s = sc[:, 8 * h + 2 * j + part]
                dl = d * (s & 0xF)
                ml = dmin * (s >> 4)
                q = (qs[:, 32 * h + 16 * part: 32 * h + 16 * part + 16] >> (2 * j)) & 3
                o = 128 * h + 32 * j + 16 * part
                out[:, o:o + 16] = dl[:, None] * q - ml[:, None]
    return out.astype(np.float32).reshape(-1)


def _q3k_scales(s12):
    """12 packed bytes -> 16 int8 scales via the kmask shuffle (gguf_dequant.py:247-264)."""
    a = np.ascontiguousarray(s12).view("<u4").reshape(-1, 3).astype(np.uint32)
    km1, km2 = np.uint32(0x03030303), np.uint32(0x0F0F0F0F)
    t = a[:, 2]
    aux = np.empty((a.shape[0], 4), dtype=np.uint32)
    aux[:, 0] = (a[:, 0] & km2) | (((t >> 0) & km1) << 4)
    aux[:, 1] = (a[:, 1] & km2) | (((t >> 2) & km1) << 4)
    aux[:, 2] = ((a[:, 0] >> 4) & km2) | (((t >> 4) & km1) << 4)
    aux[:, 3] = ((a[:, 1] >> 4) & km2) | (((t >> 6) & km1) << 4)
    return aux.view(np.int8).reshape(-1, 16).astype(np.int64)


def q3_k(raw, n):
    """gguf_dequant.py:233-293: hmask[32] @0, qs[64] @32, scales12 @96, d @108.

    Output 128h + 32j + 16p + l uses scale 8h + 2j + p, q = (qs[32h + 16p + l]
    >> 2j) & 3, minus 4 when bit (4h + j) of hmask[16p + l] is clear; value
    (d*(sc - 32)) * q (exact in float64, then one cast to float32).
    """
    b = _blocks(raw, n, 256, 110)
    nb = b.shape[0]
    hm = b[:, 0:32].astype(np.int64)
    qs = b[:, 32:96].astype(np.int64)
    sc = _q3k_scales(b[:, 96:108])
    d = _f16(b[:, 108:110]).astype(np.float64)
    out = np.empty((nb, 256), dtype=np.float64)
    for h in range(2):
        for j in range(4):
            mbit = 1 << (4 * h + j)
            for p in range(2):
                dl = d * (sc[:, 8 * h + 2 * j + p] - 32)
                q = (qs[:, 32 * h + 16 * p: 32 * h + 16 * p + 16] >> (2 * j)) & 3
                hv = np.where(hm[:, 16 * p: 16 * p + 16] & mbit, 0, 4)
                o = 128 * h + 32 * j + 16 * p
                out[:, o:o + 16] = dl[:, None] * (q - hv)
    return out.astype(np.float32).reshape(-1)


def k4_scale_min(s12):
    """(sc[8], mn[8]) 6-bit values from 12 bytes (gguf_dequant.py:299-306)."""
    s = s12.astype(np.uint32)
    sc = np.empty((s.shape[0], 8), dtype=np.uint32)
    mn = np.empty((s.shape[0], 8), dtype=np.uint32)
    for j in range(8):
        if j < 4:
            sc[:, j] = s[:, j] & 0x3F
            mn[:, j] = s[:, j + 4] & 0x3F
        else:
            sc[:, j] = (s[:, j + 4] & 0x0F) | ((s[:, j - 4] >> 6) << 4)
            mn[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
    return sc.astype(np.float32), mn.astype(np.float32)


def q4_k(raw, n):
    """gguf_dequant.py:309-341: d @0, dmin @2, scales12 @4, qs[128] @16.

    Sub-block s (32 outputs at 32s): q = (qs[32*(s//2) + l] >> 4*(s%2)) & 15;
    value (d*sc[s])*q - (dmin*mn[s]), float32, multiply then subtract.
    """
    b = _blocks(raw, n, 256, 144)
    nb = b.shape[0]
    d = _f16(b[:, 0:2])
    dmin = _f16(b[:, 2:4])
    sc, mn = k4_scale_min(b[:, 4:16])
    qs = b[:, 16:144]
    out = np.empty((nb, 256), dtype=np.float32)
    for s in range(8):
        d1 = d * sc[:, s]
        m1 = dmin * mn[:, s]
        q = ((qs[:, 32 * (s // 2): 32 * (s // 2) + 32] >> (4 * (s % 2))) & 0x0F).astype(np.float32)
        out[:, 32 * s: 32 * s + 32] = d1[:, None] * q - m1[:, None]
    return out.reshape(-1)


def q5_k(raw, n):
    """gguf_dequant.py:347-386: d @0, dmin @2, scales12 @4, qh[32] @16, qs[128] @48.

    As Q4_K, plus 16 * bit l of the little-endian u32 qh[4*(s//2) : 4*(s//2)+4]
    for element l of sub-block s (the reference's own high-bit mapping,
    gguf_dequant.py:372-381), added in float32 before the scale.
    """
    b = _blocks(raw, n, 256, 176)
    nb = b.shape[0]
    d = _f16(b[:, 0:2])
    dmin = _f16(b[:, 2:4])
    sc, mn = k4_scale_min(b[:, 4:16])
    qh = b[:, 16:48]
    qs = b[:, 48:176]
    out = np.empty((nb, 256), dtype=np.float32)
    for s in range(8):
        g = s // 2
        d1 = d * sc[:, s]
        m1 = dmin * mn[:, s]
        q = ((qs[:, 32 * g: 32 * g + 32] >> (4 * (s % 2))) & 0x0F).astype(np.float32)
        hb = _qh_bits(qh[:, 4 * g: 4 * g + 4]).astype(np.float32)
        v = q + hb * np.float32(16.0)
        out[:, 32 * s: 32 * s + 32] = d1[:, None] * v - m1[:, None]
    return out.reshape(-1)


def q6_k(raw, n):
    """gguf_dequant.py:392-436: ql[128] @0, qh[64] @128, int8 sc[16] @192, d @208.

    For half h and l < 32: outputs 128h + l + 32i (i = 0..3) take the low
    nibble of ql[64h + l] (i=0), of ql[64h + 32 + l] (i=1), the high nibbles of
    the same (i=2, 3), plus bits 2i..2i+1 of qh[32h + l] as bits 4-5; q - 32;
    value (d*sc[8h + l//16 + 2i]) * q, float32.
    """
    b = _blocks(raw, n, 256, 210)
    nb = b.shape[0]
    ql = b[:, 0:128].astype(np.int32)
    qh = b[:, 128:192].astype(np.int32)
    sc = b[:, 192:208].view(np.int8).astype(np.float32)
    d = _f16(b[:, 208:210])
    out = np.empty((nb, 256), dtype=np.float32)
    l = np.arange(32)
    for h in range(2):
        lo = ql[:, 64 * h: 64 * h + 64]
        hi = qh[:, 32 * h: 32 * h + 32]
        parts = [
            (lo[:, 0:32] & 0x0F) | (((hi >> 0) & 3) << 4),
            (lo[:, 32:64] & 0x0F) | (((hi >> 2) & 3) << 4),
            (lo[:, 0:32] >> 4) | (((hi >> 4) & 3) << 4),
            (lo[:, 32:64] >> 4) | (((hi >> 6) & 3) << 4),
        ]
        for i in range(4):
            q = (parts[i] - 32).astype(np.float32)
            s = sc[:, 8 * h + (l // 16) + 2 * i]
            out[:, 128 * h + 32 * i: 128 * h + 32 * i + 32] = (d[:, None] * s) * q
    return out.reshape(-1)


def q8_k(raw, n):
    """gguf_dequant.py:442-455: fp32 d @0, int8 qs[256] @4 (bsums @260 unused); q * d."""
    b = _blocks(raw, n, 256, 292)
    d = _f32(b[:, 0:4])
    q = b[:, 4:260].view(np.int8).astype(np.float32)
    return (q * d[:, None]).reshape(-1)


FUNCS = {
    "Q4_0": q4_0, "Q4_1": q4_1, "Q5_0": q5_0, "Q5_1": q5_1,
    "Q8_0": q8_0, "Q8_1": q8_1,
    "Q2_K": q2_k, "Q3_K": q3_k, "Q4_K": q4_k, "Q5_K": q5_k, "Q6_K": q6_k, "Q8_K": q8_k,
}


def dequant_f32(raw, name, n_elements):
    """Float32 pre-cast values of ``n_elements`` of a quantized tensor."""
    return FUNCS[name](raw, n_elements)


def _normalize(tensor_type):
    """Type-name folding of gguf_dequant.py:479-501."""
    t = tensor_type.upper()
    for p in ("Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_K"):
        if t.startswith(p):
            return p
    if t.startswith("IQ") or t.startswith("TQ"):
        raise NotImplementedError(tensor_type)
    return t


def dequantize(raw, tensor_type, shape):
    """fp16 result of the reference ``dequantize`` (gguf_dequant.py:477-523)."""
    t = _normalize(tensor_type)
    buf = np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw.view(np.uint8).reshape(-1)
    if t in ("F16", "FP16"):
        return buf.view(np.float16).reshape(shape).copy()
    if t in ("F32", "FP32"):
        return buf.view(np.float32).reshape(shape).astype(np.float16)
    if t == "BF16":
        u = buf.view(np.uint16).reshape(shape).astype(np.uint32) << 16
        return u.view(np.float32).astype(np.float16)
    plain = {"I8": np.int8, "INT8": np.int8, "I16": np.int16, "INT16": np.int16,
             "I32": np.int32, "INT32": np.int32, "I64": np.int64, "INT64": np.int64}
    if t in plain:
        return buf.view(plain[t]).reshape(shape).astype(np.float16)
    if t in FUNCS:
        n = int(np.prod(shape))
        return FUNCS[t](buf, n).reshape(shape).astype(np.float16)
    raise NotImplementedError(tensor_type)
