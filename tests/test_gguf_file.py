"""GGUF container: the parser against the reference's own parse of the same
files (tests/golden/gguf/, made by tests/golden/make_golden_gguf.py), and the
GPU loader against the oracle's dequantization of the same tensor bytes."""

import json
import os

import numpy as np
import pytest

from tests.conftest import GOLDEN
from xanosmerks_b200.gguf_file import CorruptedGGUFError, parse_gguf

GG = os.path.join(GOLDEN, "gguf")
with open(os.path.join(GG, "expected.json")) as _f:
    EXPECTED = json.load(_f)


@pytest.mark.parametrize("name", sorted(EXPECTED))
def test_parse_matches_reference(name):
    exp = EXPECTED[name]
    path = os.path.join(GG, name)
    if "error" in exp:
        cls = {"CorruptedGGUFError": CorruptedGGUFError, "EOFError": EOFError}[exp["error"]]
        with pytest.raises(cls):
            parse_gguf(path)
        return
    got = parse_gguf(path)
    assert got.pop("file") == path
    assert json.loads(json.dumps(got)) == exp["ok"]


def test_missing_file_is_corrupted_error(tmp_path):
    with pytest.raises(CorruptedGGUFError):
        parse_gguf(tmp_path / "absent.gguf")


def _tensor_bytes(info, path, t):
    start = info["data_start"] + t["offset"]
    with open(path, "rb") as f:
        f.seek(start)
        return f.read(t["size_bytes"])


@pytest.mark.gpu
@pytest.mark.parametrize("keep_quantized", [True, False])
def test_load_gguf_matches_oracle(keep_quantized):
    import torch
    from oracle import gguf_dequant_oracle as O
    from xanosmerks_b200.gguf_file import load_gguf
    from xanosmerks_b200.ops import GGUFTensor
    for fname in ("model_a.gguf", "model_b.gguf"):
        path = os.path.join(GG, fname)
        info = parse_gguf(path)
        tensors, meta = load_gguf(path, keep_quantized=keep_quantized)
        assert meta["num_tensors"] == len(info["tensors"]) and meta["metadata"] == info["metadata"]
        for t in info["tensors"]:
            raw = _tensor_bytes(info, path, t)
            with np.errstate(all="ignore"):
                ref = O.dequantize(raw, t["type"], tuple(t["shape"]))
            got = tensors[t["name"]]
            if isinstance(got, GGUFTensor):
                assert keep_quantized and got.shape == (t["shape"][1], t["shape"][0])
                got = got.dequantize().reshape(tuple(t["shape"]))
            torch.cuda.synchronize()
            g = got.cpu().numpy()
            assert g.shape == ref.shape, t["name"]
            assert np.array_equal(g.view(np.uint16), ref.astype(np.float16).view(np.uint16)), t["name"]


@pytest.mark.gpu
def test_load_gguf_unsupported_type():
    from xanosmerks_b200.gguf_file import UnsupportedDTypeError, load_gguf
    with pytest.raises(UnsupportedDTypeError):
        load_gguf(os.path.join(GG, "model_iq.gguf"))
