"""CPU: host-side behaviour of the drop-in API (no GPU needed).

The reference's dequantize dispatcher folds type names and raises
NotImplementedError for types it does not handle (gguf_dequant.py:477-523);
the replacement must do the same before touching a device.  Without a GPU the
product path must fail loudly rather than fall back to a CPU computation.
"""

import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from xanosmerks_b200 import qtypes
from xanosmerks_b200.ops import GGUFTensor, LinearOp
from xanosmerks_b200.synth import make_weight

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("name,base", [("Q4_K_M", "Q4_K"), ("q4_k_s", "Q4_K"), ("Q6_K", "Q6_K"),
                                       ("Q5_K_M", "Q5_K"), ("Q8_0", "Q8_0"), ("Q3_K_L", "Q3_K"),
                                       ("Q2_K", "Q2_K"), ("F16", "F16"), ("BF16", "BF16")])
def test_type_names_fold_like_the_reference(name, base):
    assert qtypes.normalize(name).name == base


@pytest.mark.parametrize("name", ["IQ2_XXS", "IQ4_NL", "TQ1_0", "TQ2_0", "Q9_X"])
def test_unsupported_types_raise_not_implemented(name):
    with pytest.raises(NotImplementedError):
        qtypes.normalize(name)


@pytest.mark.parametrize("name,n,k,nbytes", [("Q4_K", 11008, 4096, 25_362_432), ("Q6_K", 4096, 14336, 48_168_960),
                                             ("Q8_0", 4096, 4096, 17_825_792), ("Q5_K", 4096, 14336, 40_370_176),
                                             ("Q6_K", 4096, 4096, 13_762_560), ("Q5_K", 4096, 4096, 11_534_336)])
def test_quantized_sizes_match_the_record_layouts(name, n, k, nbytes):
    qt = qtypes.normalize(name)
    assert qtypes.row_bytes(qt, k) * n == nbytes


def test_synthetic_weights_have_the_record_sizes():
    for name, n, k in (("Q4_K", 64, 512), ("Q6_K", 32, 768), ("Q8_0", 16, 96), ("Q5_K", 8, 256)):
        raw = make_weight(name, n, k, seed=0)
        assert len(raw) == qtypes.row_bytes(qtypes.normalize(name), k) * n


def test_gguf_tensor_rejects_plain_types_before_any_device_work():
    with pytest.raises(NotImplementedError):
        GGUFTensor(b"", "F16", (1, 1))


def test_linear_op_checks_a_dense_weight_before_any_device_work():
    """A dense float weight is accepted as in the reference (LinearOp(np.eye(4)), defaults.py:109-117);
    its shape is checked on the host first."""
    with pytest.raises(ValueError):
        LinearOp(np.zeros((2, 4, 4), np.float32))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_product_path_fails_loudly_without_a_gpu():
    from xanosmerks_b200.gguf_dequant import dequantize
    raw = make_weight("Q4_K", 1, 256, seed=0)
    with pytest.raises(Exception):
        dequantize(raw, "Q4_K", (1, 256))
    with pytest.raises(Exception):
        GGUFTensor(raw, "Q4_K", (1, 256))
    with pytest.raises(Exception):
        LinearOp(np.eye(4, dtype=np.float32))


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "2", "--warmup", "1"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["dequant"]["GBps"] > 0
