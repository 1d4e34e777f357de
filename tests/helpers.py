"""Shared test helpers: golden-case iteration and comparison rules."""

import numpy as np


def golden_cases(g):
    """(key, type name, raw bytes, shape, reference fp16 bits) for every dequant fixture."""
    keys = sorted({k.rsplit("_", 1)[0] for k in g.files})
    for k in keys:
        name = k.split("_plain")[0] if "_plain" in k else "_".join(k.split("_")[:2])
        yield k, name, g[k + "_raw"], tuple(int(s) for s in g[k + "_shape"]), g[k + "_out"]


def assert_f16_bits_equal(got_bits, ref_bits, what=""):
    """Bit-for-bit fp16 equality; NaN positions must agree (payloads are not compared)."""
    got_bits = np.asarray(got_bits).view(np.uint16).reshape(-1)
    ref_bits = np.asarray(ref_bits).view(np.uint16).reshape(-1)
    assert got_bits.shape == ref_bits.shape, what
    gn = np.isnan(got_bits.view(np.float16))
    rn = np.isnan(ref_bits.view(np.float16))
    assert np.array_equal(gn, rn), f"{what}: NaN positions differ"
    bad = (got_bits != ref_bits) & ~rn
    if bad.any():
        i = int(np.flatnonzero(bad)[0])
        raise AssertionError(f"{what}: {int(bad.sum())} elements differ; first at {i}: "
                             f"got {got_bits[i]:#06x} ref {ref_bits[i]:#06x}")


def assert_f32_bits_equal(got, ref, what=""):
    got = np.asarray(got, dtype=np.float32).reshape(-1)
    ref = np.asarray(ref, dtype=np.float32).reshape(-1)
    gn, rn = np.isnan(got), np.isnan(ref)
    assert np.array_equal(gn, rn), f"{what}: NaN positions differ"
    bad = (got.view(np.uint32) != ref.view(np.uint32)) & ~rn
    if bad.any():
        i = int(np.flatnonzero(bad)[0])
        raise AssertionError(f"{what}: {int(bad.sum())} elements differ; first at {i}: got {got[i]!r} ref {ref[i]!r}")


def rel_err(got, ref):
    """Normwise relative error max|got - ref| / max|ref| (the matmul tolerance metric)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(got - ref)) / (den if den > 0 else 1.0))


# Matmul tolerances (normwise, fp32 accumulation): the decode GEMV on fp32
# activations and the prefill GEMM.
GEMV_TOL = 1e-3
GEMM_TOL = 2e-3
