"""CPU oracle for the MoE block and the linear ops -- test infrastructure only.

Restates moe.py:54-115 (``MoELayer.__call__``) and ops.py:55-67
(``LinearOp.forward``) in numpy, on already-dequantized fp32 weights.  Imported
only by tests, ``smoke()`` and the CPU-baseline leg of ``bench.py``.
"""

from __future__ import annotations

import numpy as np


def softmax(x, axis=-1):
    """primitives.py:7-11 (the fallback the reference uses without ninewas9)."""
    x_max = np.max(x, axis=axis, keepdims=True)
    x_max = np.where(np.isfinite(x_max), x_max, 0.0)
    e = np.exp(x - x_max)
    return e / (np.sum(e, axis=axis, keepdims=True) + 1e-12)


def silu(x):
    """primitives.py:37-39."""
    return x / (1.0 + np.exp(-x))


def gelu(x):
    """primitives.py:47-49 (tanh form)."""
    return 0.5 * x * (1.0 + np.tanh(0.7978845608 * (x + 0.044715 * x ** 3)))


def relu(x):
    """primitives.py:58-59."""
    return np.maximum(x, 0.0)


def identity(x):
    """primitives.py:60-61."""
    return x


# apply_activation's names (primitives.py:52-62)
ACTS = {"silu": silu, "swish": silu, "gelu": gelu, "relu": relu, "identity": identity}


def expert_ffn(xs, w1, w3, w2, act=silu):
    """One expert on its rows (moe.py:106-109): act(xs @ w1.T) * (xs @ w3.T) @ w2.T."""
    return (act(xs @ w1.T) * (xs @ w3.T)) @ w2.T


def linear(x, w, b=None):
    """ops.py:62-67: fp32(x) @ W.T (+ b)."""
    y = np.asarray(x, dtype=np.float32) @ np.asarray(w, dtype=np.float32).T
    return y + b if b is not None else y


def route(logits, k):
    """Top-k experts and their softmax weights (moe.py:75-81), plus the stable
    expert-major dispatch order (moe.py:83-93)."""
    n_tok, n_exp = logits.shape
    if k == n_exp:
        return None
    top = np.argpartition(-logits, k - 1, axis=-1)[:, :k]
    top_logits = np.take_along_axis(logits, top, axis=-1)
    w = softmax(top_logits, axis=-1)
    flat_e = top.reshape(-1)
    flat_w = w.reshape(-1)
    flat_t = np.repeat(np.arange(n_tok), k)
    order = np.argsort(flat_e, kind="stable")
    counts = np.bincount(flat_e[order], minlength=n_exp)
    return flat_e[order], flat_w[order], flat_t[order], counts


def moe_forward(x, gate_w, experts, k, act=silu):
    """moe.py:54-115 on fp32 weights; experts[i] = {"w1": (F,H), "w3": (F,H), "w2": (H,F)}."""
    b, s, h = x.shape
    xf = x.reshape(-1, h)
    logits = xf @ np.asarray(gate_w, dtype=np.float32).T
    out = np.zeros_like(xf)
    n_exp = len(experts)
    if k == n_exp:
        wts = softmax(logits, axis=-1)
        for e in range(n_exp):
            out += expert_ffn(xf, experts[e]["w1"], experts[e]["w3"], experts[e]["w2"], act) * wts[:, e:e + 1]
        return out.reshape(b, s, h)
    se, sw, st, counts = route(logits, k)
    start = 0
    for e in range(n_exp):
        end = start + int(counts[e])
        if end > start:
            tok = st[start:end]
            y = expert_ffn(xf[tok], experts[e]["w1"], experts[e]["w3"], experts[e]["w2"], act)
            out[tok] += y * sw[start:end, None]
        start = end
    return out.reshape(b, s, h)


def combine(n_tok, h, routing, expert_out):
    """The scatter-add of moe.py:110-113 given each expert's output rows in dispatch order:
    ``routing`` = route(...), ``expert_out[e]`` = that expert's rows (ascending expert order)."""
    se, sw, st, counts = routing
    out = np.zeros((n_tok, h), dtype=np.float32)
    start = 0
    for e in range(len(counts)):
        end = start + int(counts[e])
        if end > start:
            out[st[start:end]] += expert_out[e] * sw[start:end, None]
        start = end
    return out
