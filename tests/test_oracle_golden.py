"""CPU: the oracle restatement reproduces the reference's own outputs (golden fixtures)."""

import json
import os

import numpy as np
import pytest

from oracle import gguf_dequant_oracle as O
from tests.conftest import GOLDEN
from tests.helpers import assert_f16_bits_equal, golden_cases, rel_err


def test_golden_covers_every_type(golden_dequant):
    names = {c[1] for c in golden_cases(golden_dequant)}
    assert names >= set(O.FUNCS) | {"F16", "F32", "BF16", "I8", "I16", "I32", "I64"}


def test_oracle_dequant_bit_exact(golden_dequant):
    n = 0
    for key, name, raw, shape, ref in golden_cases(golden_dequant):
        with np.errstate(all="ignore"):
            got = O.dequantize(raw.tobytes(), name, shape)
        assert got.shape == shape
        assert_f16_bits_equal(got, ref, key)
        n += 1
    assert n >= 55


def test_oracle_names(tmp_path):
    with open(os.path.join(GOLDEN, "golden_names.json")) as f:
        names = json.load(f)
    from xanosmerks_b200 import qtypes
    for nm, outcome in names.items():
        if outcome == "NotImplementedError":
            with pytest.raises(NotImplementedError):
                qtypes.normalize(nm)
        else:
            qtypes.normalize(nm)


def test_oracle_linear(golden_linear):
    g = golden_linear
    for name in ("Q4_K", "Q6_K", "Q8_0", "Q5_K", "Q4_0"):
        n, k = (int(v) for v in g[f"{name}_nk"])
        w = O.dequantize(g[f"{name}_raw"].tobytes(), name, (n, k)).astype(np.float32)
        for m in (1, 3, 8):
            y = g[f"{name}_m{m}_x"] @ w.T
            assert rel_err(y, g[f"{name}_m{m}_y"]) < 1e-6
        x = g[f"{name}_bias_x"]
        assert rel_err(x @ w.T + g[f"{name}_bias_b"], g[f"{name}_bias_y"]) < 1e-6


def test_oracle_moe(golden_moe):
    from oracle.moe_oracle import moe_forward
    g = golden_moe
    E, H, F = (int(v) for v in g["ehf"])
    experts = []
    for e in range(E):
        ws = {}
        for wn, (r, c) in (("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F))):
            ws[wn] = O.dequantize(g[f"raw_e{e}_{wn}"].tobytes(), "Q4_K", (r, c)).astype(np.float32)
        experts.append(ws)
    for k in (1, 2, E):
        y = moe_forward(g["x"], g["gate_w"], experts, k)
        assert rel_err(y, g[f"y_k{k}"]) < 1e-5, k
