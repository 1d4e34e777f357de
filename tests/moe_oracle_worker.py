"""Oracle work for the full-size MoE parity test, run in spawned worker processes:
one expert's weights dequantized by the oracle (gguf_dequant.py's unpackers
restated in numpy) and its FFN on the rows routed to it (moe.py:106-109)."""

import numpy as np


def expert_rows(args):
    """(raw w1, raw w3, raw w2, qtype, H, F, rows of x, activation name) -> fp32 output rows."""
    raw1, raw3, raw2, qtype, H, F, xs, act = args
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(2)
    except ImportError:
        pass
    from oracle import gguf_dequant_oracle as O
    from oracle.moe_oracle import ACTS, expert_ffn
    w1 = O.dequantize(raw1, qtype, (F, H)).astype(np.float32)
    w3 = O.dequantize(raw3, qtype, (F, H)).astype(np.float32)
    w2 = O.dequantize(raw2, qtype, (H, F)).astype(np.float32)
    if xs.shape[0] == 0:
        return np.zeros((0, H), np.float32)
    return expert_ffn(xs, w1, w3, w2, ACTS[act]).astype(np.float32)
