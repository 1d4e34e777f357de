"""Host-side logic of the decoder (CPU): tensor-parallel sharding of GGUF
weights keeps the bytes of each row's K-slice / each row block, and the
shards of all ranks reassemble the full matrix."""

import numpy as np
import torch

from oracle import gguf_dequant_oracle as O
from xanosmerks_b200.llama import LlamaConfig, _cat_rows, shard_cols, shard_rows
from xanosmerks_b200.ops import GGUFTensor
from xanosmerks_b200.synth import make_weight


class _HostTensor(GGUFTensor):
    """GGUFTensor over host memory (the sharding helpers only slice bytes)."""

    def __init__(self, raw, name, shape):
        from xanosmerks_b200 import qtypes
        self.qtype = qtypes.normalize(name)
        self.shape = tuple(shape)
        self.data = torch.as_tensor(raw).view(torch.uint8).reshape(-1)


def test_shard_cols_and_rows_reassemble(monkeypatch):
    import xanosmerks_b200.llama as L
    monkeypatch.setattr(L, "GGUFTensor", _HostTensor)
    for name, n, k, world in (("Q6_K", 64, 14336, 8), ("Q4_K", 48, 4096, 4), ("Q8_0", 16, 1024, 2)):
        raw = make_weight(name, n, k, seed=1)
        full = O.dequantize(raw, name, (n, k)).astype(np.float32)
        t = _HostTensor(raw, name, (n, k))
        cols = [L.shard_cols(t, r * k // world, (r + 1) * k // world) for r in range(world)]
        got = np.concatenate([O.dequantize(c.data.numpy().tobytes(), name, c.shape).astype(np.float32)
                              for c in cols], axis=1)
        assert np.array_equal(got.view(np.uint32), full.view(np.uint32)), name
        rows = [L.shard_rows(t, r * n // world, (r + 1) * n // world) for r in range(world)]
        cat = L._cat_rows(rows)
        assert np.array_equal(cat.data.numpy(), raw)


def test_config_bytes_per_token():
    cfg = LlamaConfig()
    # Q4_K attention + gate/up, Q6_K down and output: 32 x 137.8 MB + 107.5 MB
    assert cfg.weight_bytes_per_token() == 32 * (6144 * 2304 + 4096 * 2304 + 28672 * 2304 + 4096 * 56 * 210) \
        + 32000 * 16 * 210
    ref = cfg.reference_config()
    assert ref["num_kv_heads"] == 8 and ref["rope_theta"] == 5e5 and ref["norm_eps"] == 1e-5
