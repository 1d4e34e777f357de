"""Seeded synthetic GGUF blocks (weights are random-init; no model file is needed).

Records are built byte-wise: every byte uniform random, then the scale fields
overwritten with the value distribution asked for.  The ``"config"`` layout
follows the synthetic workloads this library is measured on:

* Q8_0: fp16 ``d = |N(0,1)| * 0.02``, 32 int8 uniform in [-127, 127];
* Q4_K: fp16 ``d, dmin = |N(0,1)| * 0.01``, random scale and nibble bytes;
* Q6_K: random ql/qh/scales, fp16 ``d = |N(0,1)| * 0.005``;
* Q5_K: ``d, dmin`` as Q4_K, random scales/qh/qs;

and, for the formats no workload names, the same idea (``|N| * 0.01`` scales,
``N * 0.01`` offsets, random payload bytes).  ``"random"`` leaves every byte
random (so scale fields include fp16 inf/NaN patterns) and ``"edge"`` plants
extreme scale values: subnormals, the fp16 maximum, zero, negatives and fp32
values that overflow or underflow fp16.
"""

from __future__ import annotations

import numpy as np

RECORD = {"Q4_0": 18, "Q4_1": 20, "Q5_0": 22, "Q5_1": 24, "Q8_0": 34, "Q8_1": 40,
          "Q2_K": 84, "Q3_K": 110, "Q4_K": 144, "Q5_K": 176, "Q6_K": 210, "Q8_K": 292}
QK = {n: (32 if RECORD[n] <= 40 else 256) for n in RECORD}

# (byte offset, kind, config distribution): kind "f16"/"f32"; dist ("abs", s) = |N|*s,
# ("n", s) = N*s.  Offsets follow the record layouts of the reference's unpackers.
_FIELDS = {
    "Q4_0": [(0, "f16", ("abs", 0.01))],
    "Q4_1": [(0, "f16", ("abs", 0.01)), (2, "f16", ("n", 0.01))],
    "Q5_0": [(0, "f16", ("abs", 0.01))],
    "Q5_1": [(0, "f16", ("abs", 0.01)), (2, "f16", ("n", 0.01))],
    "Q8_0": [(0, "f16", ("abs", 0.02))],
    "Q8_1": [(0, "f32", ("abs", 0.02)), (4, "f32", ("n", 0.01))],
    "Q2_K": [(80, "f16", ("abs", 0.01)), (82, "f16", ("abs", 0.01))],
    "Q3_K": [(108, "f16", ("abs", 0.01))],
    "Q4_K": [(0, "f16", ("abs", 0.01)), (2, "f16", ("abs", 0.01))],
    "Q5_K": [(0, "f16", ("abs", 0.01)), (2, "f16", ("abs", 0.01))],
    "Q6_K": [(208, "f16", ("abs", 0.005))],
    "Q8_K": [(0, "f32", ("abs", 0.01))],
}

_EDGE_F16 = np.array([0x0001, 0x03FF, 0x0400, 0x7BFF, 0x0000, 0x8000, 0xBC00, 0x3C00,
                      0x5BFF, 0x1234, 0xFBFF, 0x2E66], dtype=np.uint16)
_EDGE_F32 = np.array([1e30, -1e30, 1e-30, 0.0, -0.0, 1.0, 65504.0, 70000.0, 3e-8,
                      -2.5, 1.1754944e-38, 0.02], dtype=np.float32)


def make_blocks(name: str, n_blocks: int, rng: np.random.Generator, dist: str = "config") -> np.ndarray:
    """``n_blocks`` records of qtype ``name`` as a flat uint8 array."""
    rec = RECORD[name]
    b = rng.integers(0, 256, size=(n_blocks, rec), dtype=np.uint8)
    if name == "Q8_0" and dist == "config":
        b[:, 2:34] = rng.integers(-127, 128, size=(n_blocks, 32), dtype=np.int8).view(np.uint8)
    if dist == "random":
        return b.reshape(-1)
    for off, kind, (mode, scale) in _FIELDS[name]:
        if dist == "edge":
            if kind == "f16":
                v = rng.choice(_EDGE_F16, size=n_blocks).astype(np.uint16)
            else:
                v = rng.choice(_EDGE_F32, size=n_blocks).astype(np.float32).view(np.uint32)
        else:
            g = rng.standard_normal(n_blocks)
            g = np.abs(g) * scale if mode == "abs" else g * scale
            v = g.astype(np.float16).view(np.uint16) if kind == "f16" else g.astype(np.float32).view(np.uint32)
        w = 2 if kind == "f16" else 4
        b[:, off:off + w] = np.ascontiguousarray(v).view(np.uint8).reshape(n_blocks, w)
    return b.reshape(-1)


def make_weight(name: str, n: int, k: int, seed: int = 0, dist: str = "config") -> np.ndarray:
    """Row-major (n rows x k elements) quantized weight as flat GGUF bytes."""
    if k % QK[name]:
        raise ValueError(f"{name}: k={k} is not a multiple of {QK[name]}")
    rng = np.random.default_rng(seed)
    return make_blocks(name, n * k // QK[name], rng, dist)


def make_weight_device(name: str, n: int, k: int, seed: int = 0, device="cuda", scale: float | None = None):
    """The ``"config"`` distribution of :func:`make_weight` generated on the GPU
    (torch generator, so a 4.5 GB model takes a second rather than minutes):
    a flat uint8 CUDA tensor of ``n * k / QK * record`` bytes.  ``scale``
    replaces the distribution's scale factor of every fp16/fp32 scale field
    (``|N(0,1)| * scale``), e.g. to give a decoder layer weights of a trained
    model's magnitude.  The bytes differ from :func:`make_weight` for the same
    seed (a different generator); copy them to the host to check them."""
    import torch

    if k % QK[name]:
        raise ValueError(f"{name}: k={k} is not a multiple of {QK[name]}")
    rec = RECORD[name]
    nb = n * k // QK[name]
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    b = torch.randint(0, 256, (nb, rec), dtype=torch.uint8, device=device, generator=g)
    if name == "Q8_0":
        q = torch.randint(-127, 128, (nb, 32), dtype=torch.int16, device=device, generator=g)
        b[:, 2:34] = q.to(torch.int8).view(torch.uint8)
    for off, kind, (mode, s) in _FIELDS[name]:
        s = s if scale is None else scale
        v = torch.randn(nb, device=device, generator=g, dtype=torch.float32)
        v = v.abs() * s if mode == "abs" else v * s
        if kind == "f16":
            b[:, off:off + 2] = v.to(torch.float16).view(torch.uint8).reshape(nb, 2)
        else:
            b[:, off:off + 4] = v.view(torch.uint8).reshape(nb, 4)
    return b.reshape(-1)
