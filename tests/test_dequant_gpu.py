"""GPU parity: the CUDA dequant kernels reproduce the reference bit for bit.

Checked against the reference's own outputs (golden fixtures) and, at larger
and full sizes, against the oracle restatement on seeded inputs.
"""

import numpy as np
import pytest
import torch

from oracle import gguf_dequant_oracle as O
from tests.helpers import assert_f16_bits_equal, assert_f32_bits_equal, golden_cases
from xanosmerks_b200 import gguf_dequant as G
from xanosmerks_b200 import qtypes
from xanosmerks_b200.synth import QK, RECORD, make_blocks

pytestmark = pytest.mark.gpu

QUANT = list(RECORD)


def test_golden_fixtures_host_api(golden_dequant):
    """Every reference fixture through the host (numpy in, numpy out) entry point."""
    for key, name, raw, shape, ref in golden_cases(golden_dequant):
        got = G.dequantize(raw.tobytes(), name, shape)
        assert isinstance(got, np.ndarray) and got.dtype == np.float16 and got.shape == shape
        assert_f16_bits_equal(got, ref, key)


def test_golden_fixtures_per_type_functions(golden_dequant):
    for key, name, raw, shape, ref in golden_cases(golden_dequant):
        if name in G.DEQUANT_FUNCS:
            assert_f16_bits_equal(G.DEQUANT_FUNCS[name](raw.tobytes(), shape), ref, key)


@pytest.mark.parametrize("name", QUANT)
@pytest.mark.parametrize("dist", ["config", "random", "edge"])
def test_seeded_vs_oracle_fp16_and_fp32(name, dist):
    rng = np.random.default_rng(hash((name, dist)) % 2**32)
    nblk = 4099 if QK[name] == 32 else 517          # ragged: not a multiple of any CTA tile
    raw = make_blocks(name, nblk, rng, dist)
    n = nblk * QK[name]
    d_raw = torch.from_numpy(raw).cuda()
    got16 = G.dequantize(d_raw, name, (n,)).cpu().numpy()
    got32 = G.dequantize(d_raw, name, (n,), out_dtype="float32").cpu().numpy()
    with np.errstate(all="ignore"):
        ref32 = O.dequant_f32(raw, name, n)
        ref16 = ref32.astype(np.float16)
    assert_f16_bits_equal(got16, ref16, f"{name}/{dist} fp16")
    assert_f32_bits_equal(got32, ref32, f"{name}/{dist} fp32")


@pytest.mark.parametrize("name", QUANT)
@pytest.mark.parametrize("offset", [1, 2, 3, 8, 15])
def test_unaligned_input_pointer(name, offset):
    """Blocks starting at any byte offset (e.g. a tensor inside an mmapped file)."""
    rng = np.random.default_rng(offset)
    nblk = 37
    raw = make_blocks(name, nblk, rng, "config")
    buf = np.zeros(raw.size + 64, np.uint8)
    buf[offset:offset + raw.size] = raw
    d = torch.from_numpy(buf).cuda()[offset:offset + raw.size]
    n = nblk * QK[name]
    got = G.dequantize(d, name, (n,)).cpu().numpy()
    assert_f16_bits_equal(got, O.dequant_f32(raw, name, n).astype(np.float16), f"{name}+{offset}")


@pytest.mark.parametrize("name,shape", [("Q8_0", (4096, 4096)), ("Q4_K", (11008, 4096)),
                                        ("Q6_K", (4096, 14336)), ("Q5_K", (4096, 14336))])
def test_full_config_sizes(name, shape):
    raw = make_blocks(name, shape[0] * shape[1] // QK[name], np.random.default_rng(0), "config")
    got = G.dequantize(torch.from_numpy(raw).cuda(), name, shape)
    assert got.shape == shape
    ref = O.dequant_f32(raw, name, shape[0] * shape[1]).astype(np.float16)
    assert_f16_bits_equal(got.cpu().numpy(), ref, name)


def test_plain_types_and_errors():
    x = np.random.default_rng(3).standard_normal(96).astype(np.float32) * 3e4
    got = G.dequantize(x.tobytes(), "F32", (8, 12))
    assert_f16_bits_equal(got, x.reshape(8, 12).astype(np.float16))
    with pytest.raises(NotImplementedError):
        G.dequantize(b"\0" * 66, "IQ2_XXS", (256,))
    with pytest.raises(NotImplementedError):
        G.dequantize(b"\0" * 66, "TQ2_0", (256,))
    with pytest.raises(ValueError):
        G.dequantize(b"\0" * 143, "Q4_K", (256,))     # truncated buffer
    with pytest.raises(ValueError):
        G.dequantize(b"\0" * 288, "Q4_K", (300,))     # not a multiple of the block
    with pytest.raises(ValueError):
        G.dequantize(b"\0" * 10, "F16", (4,))         # plain types need the exact size
    assert G.dequantize(b"", "Q4_K", (0,)).shape == (0,)
    # extra trailing bytes are ignored, as in the reference
    raw = make_blocks("Q8_0", 3, np.random.default_rng(1), "config")
    got = G.dequantize(raw.tobytes() + b"\1" * 7, "q8_0", (96,))
    assert_f16_bits_equal(got, O.dequantize(raw.tobytes(), "Q8_0", (96,)))
    # Q4_K_M-style names fold to the base K-quant
    raw = make_blocks("Q4_K", 2, np.random.default_rng(2), "config")
    assert_f16_bits_equal(G.dequantize(raw.tobytes(), "Q4_K_M", (2, 256)), O.dequantize(raw.tobytes(), "Q4_K", (2, 256)))
