"""Generate the golden fixtures in this folder by running the reference itself.

Run (in a checkout that has the reference's sources available):

    python tests/golden/make_golden.py --reference <path to the reference package sources>

It builds a throwaway package of symlinks to the reference's hot-path modules
(gguf_dequant.py, dtype_ops.py, ops.py, primitives.py, moe.py) so their relative
imports resolve, feeds them seeded synthetic inputs, and writes:

* ``golden_dequant.npz`` -- raw GGUF block bytes, shape and the reference's fp16
  output (as uint16 bit patterns) for every quantized type and plain type;
* ``golden_names.json``  -- how the reference dispatcher treats type names;
* ``golden_linear.npz``  -- ``LinearOp`` / ``FusedRMSNormLinearOp`` / SwiGLU-MLP
  outputs on dequantized weights;
* ``golden_moe.npz``     -- ``MoELayer`` outputs (sparse top-2 and dense).

The fixtures are committed; nothing at test time reads the reference.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from xanosmerks_b200.synth import make_blocks, RECORD, QK  # noqa: E402

MODULES = ["gguf_dequant", "dtype_ops", "ops", "primitives", "moe"]


def load_reference(ref_dir):
    tmp = tempfile.mkdtemp(prefix="xmref_")
    pkg = os.path.join(tmp, "xmref")
    os.makedirs(pkg)
    open(os.path.join(pkg, "__init__.py"), "w").close()
    for m in MODULES:
        os.symlink(os.path.join(ref_dir, m + ".py"), os.path.join(pkg, m + ".py"))
    sys.path.insert(0, tmp)
    return {m: importlib.import_module("xmref." + m) for m in MODULES}


def dequant_cases(ref):
    gd = ref["gguf_dequant"]
    out = {}
    rng = np.random.default_rng(1234)
    for name in RECORD:
        qk = QK[name]
        cases = [
            ("cfg", (2, 4 * qk), "config"),
            ("rand", (16 * qk,), "random"),
            ("edge", (2, 2, 2 * qk), "edge"),
            ("one", (qk,), "config"),
        ]
        for tag, shape, dist in cases:
            n_el = int(np.prod(shape))
            raw = make_blocks(name, n_el // qk, rng, dist)
            y = gd.dequantize(raw.tobytes(), name, shape)
            assert y.dtype == np.float16 and y.shape == shape
            key = f"{name}_{tag}"
            out[key + "_raw"] = raw
            out[key + "_shape"] = np.array(shape, dtype=np.int64)
            out[key + "_out"] = y.view(np.uint16)
    # plain passthrough types (gguf_dequant.py:503-518)
    plain = {
        "F16": rng.standard_normal(64).astype(np.float16).view(np.uint8),
        "F32": np.concatenate([rng.standard_normal(60).astype(np.float32) * 1000,
                               np.array([65519.99, 65520.0, 3e-8, -1e-9], np.float32)]).view(np.uint8),
        "BF16": (rng.standard_normal(64).astype(np.float32) * 100).view(np.uint32).__rshift__(16).astype(np.uint16).view(np.uint8),
        "I8": rng.integers(-128, 128, 64).astype(np.int8).view(np.uint8),
        "I16": rng.integers(-32768, 32768, 64).astype(np.int16).view(np.uint8),
        "I32": np.concatenate([rng.integers(-70000, 70000, 60), [2049, 65519, 65520, -65520]]).astype(np.int32).view(np.uint8),
        "I64": np.concatenate([rng.integers(-70000, 70000, 60), [2049, 2**40 + 1, -(2**33), 4097]]).astype(np.int64).view(np.uint8),
    }
    for name, raw in plain.items():
        shape = (4, 16)
        y = gd.dequantize(raw.tobytes(), name, shape)
        out[f"{name}_plain_raw"] = raw
        out[f"{name}_plain_shape"] = np.array(shape, dtype=np.int64)
        out[f"{name}_plain_out"] = y.view(np.uint16)
    return out


def name_cases(ref):
    """Outcome of the reference dispatcher for a list of type names."""
    gd = ref["gguf_dequant"]
    names = ["q4_k_m", "Q4_K_S", "Q5_K_M", "q6_k", "Q3_K_L", "Q2_K_S", "Q8_K", "q8_0",
             "Q4_0", "q5_1", "fp16", "F32", "bf16", "int8", "I64",
             "IQ2_XXS", "iq4_nl", "TQ1_0", "tq2_0", "Q9_9", "F64", "U8"]
    res = {}
    for nm in names:
        buf = np.zeros(256 * 8, np.uint8)   # enough bytes for 256 elements of any type
        try:
            y = gd.dequantize(buf.tobytes(), nm, (256,) if not nm.upper().startswith(("F", "BF", "I", "INT")) else (buf.size // {"F16": 2, "FP16": 2, "BF16": 2, "F32": 4, "I64": 8, "INT8": 1, "F64": 8}.get(nm.upper(), 1),))
            res[nm] = f"ok:{y.dtype}"
        except NotImplementedError:
            res[nm] = "NotImplementedError"
        except Exception as e:  # noqa: BLE001
            res[nm] = type(e).__name__
    return res


def linear_cases(ref):
    gd, ops, prim = ref["gguf_dequant"], ref["ops"], ref["primitives"]
    rng = np.random.default_rng(77)
    out = {}
    for name, (n, k) in {"Q4_K": (48, 512), "Q6_K": (40, 512), "Q8_0": (36, 256),
                         "Q5_K": (32, 512), "Q4_0": (24, 128)}.items():
        raw = make_blocks(name, n * k // QK[name], rng, "config")
        w = gd.dequantize(raw.tobytes(), name, (n, k))
        for m in (1, 3, 8):
            x = rng.standard_normal((m, k)).astype(np.float32)
            y = ops.LinearOp(w).forward(x)
            out[f"{name}_m{m}_x"] = x
            out[f"{name}_m{m}_y"] = y
        b = rng.standard_normal(n).astype(np.float32)
        x = rng.standard_normal((2, 3, k)).astype(np.float32)
        out[f"{name}_bias_b"] = b
        out[f"{name}_bias_x"] = x
        out[f"{name}_bias_y"] = ops.LinearOp(w, b).forward(x)
        nw = (1 + 0.1 * rng.standard_normal(k)).astype(np.float32)
        out[f"{name}_rms_nw"] = nw
        out[f"{name}_rms_y"] = ops.FusedRMSNormLinearOp(nw, w).forward(x)
        out[f"{name}_raw"] = raw
        out[f"{name}_nk"] = np.array([n, k], dtype=np.int64)
    # SwiGLU MLP in the composition of forward.py:93-103 (gate/up Q4_K, down Q6_K)
    h, f = 256, 512
    rg = make_blocks("Q4_K", f * h // 256, rng, "config")
    ru = make_blocks("Q4_K", f * h // 256, rng, "config")
    rd = make_blocks("Q6_K", h * f // 256, rng, "config")
    wg = gd.dequantize(rg.tobytes(), "Q4_K", (f, h)).astype(np.float32)
    wu = gd.dequantize(ru.tobytes(), "Q4_K", (f, h)).astype(np.float32)
    wd = gd.dequantize(rd.tobytes(), "Q6_K", (h, f)).astype(np.float32)
    x = rng.standard_normal((1, 4, h)).astype(np.float32)
    gate = x @ wg.T
    up = x @ wu.T
    y = prim.swiglu(gate, up) @ wd.T
    out.update(mlp_gate_raw=rg, mlp_up_raw=ru, mlp_down_raw=rd, mlp_x=x, mlp_y=y,
               mlp_hf=np.array([h, f], dtype=np.int64))
    return out


def moe_cases(ref):
    gd, moe = ref["gguf_dequant"], ref["moe"]
    rng = np.random.default_rng(99)
    out = {}
    E, H, F = 4, 256, 256
    gate_w = rng.standard_normal((E, H)).astype(np.float32) * 0.05
    raws = {}
    weights = {"gate": {"weight": gate_w}, "experts": {}}
    for e in range(E):
        ew = {}
        for wn, (rows, cols) in (("w1", (F, H)), ("w3", (F, H)), ("w2", (H, F))):
            raw = make_blocks("Q4_K", rows * cols // 256, rng, "config")
            raws[f"e{e}_{wn}"] = raw
            ew[wn] = {"weight": gd.dequantize(raw.tobytes(), "Q4_K", (rows, cols))}
        weights["experts"][str(e)] = ew
    x = rng.standard_normal((2, 5, H)).astype(np.float32)
    for k in (1, 2, E):
        layer = moe.MoELayer({"num_experts": E, "num_experts_per_tok": k, "hidden_act": "silu"}, weights)
        out[f"y_k{k}"] = layer(x)
    out.update({f"raw_{kk}": v for kk, v in raws.items()})
    out.update(gate_w=gate_w, x=x, ehf=np.array([E, H, F], dtype=np.int64))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("XM_REFERENCE_DIR"), required="XM_REFERENCE_DIR" not in os.environ,
                    help="directory holding the reference modules (or set XM_REFERENCE_DIR)")
    args = ap.parse_args()
    ref = load_reference(args.reference)
    np.savez_compressed(os.path.join(HERE, "golden_dequant.npz"), **dequant_cases(ref))
    with open(os.path.join(HERE, "golden_names.json"), "w") as f:
        json.dump(name_cases(ref), f, indent=1, sort_keys=True)
    np.savez_compressed(os.path.join(HERE, "golden_linear.npz"), **linear_cases(ref))
    np.savez_compressed(os.path.join(HERE, "golden_moe.npz"), **moe_cases(ref))
    for fn in sorted(os.listdir(HERE)):
        print(fn, os.path.getsize(os.path.join(HERE, fn)))


if __name__ == "__main__":
    main()
