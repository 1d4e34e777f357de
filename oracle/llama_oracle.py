"""CPU oracle for the Llama decoder step -- test infrastructure only.

A numpy restatement of the reference's ``TransformerModel`` forward with a KV
cache (forward.py:19-160, attention.py:7-115, primitives.py:20-44) on
already-dequantized fp32 weights.  Imported only by tests, ``smoke()`` and the
CPU-baseline leg of ``bench.py``.

Parity: the projections, RMSNorm, SwiGLU and residual structure follow the
reference line by line and are pinned through ``LinearOp`` /
``FusedRMSNormLinearOp`` golden fixtures.  The rotary embedding, the KV cache
and ``scaled_dot_product_attention`` come from the third-party ``ninewas9``
package (PyPI ``9was9>=0.1.1``, pyproject.toml:16), which is not present, so
those three are restated from their call sites (attention.py:59-115) and the
standard definitions -- rotate-half RoPE with inv_freq = theta^(-2i/d), a cache
indexed [layer, batch, kv_head, position, dim], softmax(q k^T / sqrt(d) +
causal mask) v with query head h reading KV head h // (Hq / Hk) -- and are
**parity unpinned**.
"""

from __future__ import annotations

import numpy as np


def rms_norm(x, w, eps):
    """primitives.py:20-23."""
    rms = np.sqrt(np.mean(x ** 2, axis=-1, keepdims=True) + eps)
    return (x / rms) * w


def silu(x):
    """primitives.py:37-39."""
    return x / (1.0 + np.exp(-x))


def softmax(x, axis=-1):
    """primitives.py:7-11."""
    x_max = np.max(x, axis=axis, keepdims=True)
    x_max = np.where(np.isfinite(x_max), x_max, 0.0)
    e = np.exp(x - x_max)
    return e / (np.sum(e, axis=axis, keepdims=True) + 1e-12)


def rope(x, positions, theta):
    """Rotate-half rotary embedding of x [B, H, S, D] at positions [S]."""
    d = x.shape[-1]
    inv_freq = (1.0 / (theta ** (np.arange(0, d, 2, dtype=np.float32) / np.float32(d)))).astype(np.float32)
    ang = np.asarray(positions, dtype=np.float32)[:, None] * inv_freq[None, :]        # [S, D/2]
    cos = np.concatenate([np.cos(ang), np.cos(ang)], axis=-1).astype(np.float32)
    sin = np.concatenate([np.sin(ang), np.sin(ang)], axis=-1).astype(np.float32)
    half = d // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return x * cos + rot * sin


class LlamaOracle:
    """Decoder with an fp32 KV cache.  ``weights``: ``embed`` [V, D],
    ``layers`` (list of dicts wq, wk, wv, wo, wg, wu, wd, n1, n2), ``norm``,
    ``lm_head``; all fp32 numpy (dequantized from the same GGUF blocks)."""

    def __init__(self, cfg, weights, batch, max_ctx):
        self.cfg = cfg
        self.w = weights
        L, Hk, D = cfg["num_layers"], cfg["num_kv_heads"], cfg["head_dim"]
        self.k = np.zeros((L, batch, Hk, max_ctx, D), dtype=np.float32)
        self.v = np.zeros_like(self.k)

    def _attn(self, layer, x, pos):
        """attention.py:39-115 (fused_qkv, RoPE, cache append, causal SDPA, o_proj)."""
        c, w = self.cfg, self.w["layers"][layer]
        B, S, _ = x.shape
        Hq, Hk, D = c["num_heads"], c["num_kv_heads"], c["head_dim"]
        q = (x @ w["wq"].T).reshape(B, S, Hq, D).transpose(0, 2, 1, 3)
        k = (x @ w["wk"].T).reshape(B, S, Hk, D).transpose(0, 2, 1, 3)
        v = (x @ w["wv"].T).reshape(B, S, Hk, D).transpose(0, 2, 1, 3)
        positions = np.arange(pos, pos + S)
        q = rope(q, positions, c["rope_theta"])
        k = rope(k, positions, c["rope_theta"])
        self.k[layer, :, :, pos:pos + S] = k
        self.v[layer, :, :, pos:pos + S] = v
        kv = pos + S
        kf, vf = self.k[layer, :, :, :kv], self.v[layer, :, :, :kv]
        r = Hq // Hk
        qg = q.reshape(B, Hk, r, S, D)
        scores = np.matmul(qg, np.swapaxes(kf[:, :, None], -1, -2)) / np.float32(np.sqrt(D))
        if S > 1:
            mask = np.full((S, kv), -np.inf, dtype=np.float32)
            for i in range(S):
                mask[i, :pos + i + 1] = 0.0
            scores = scores + mask
        out = np.matmul(softmax(scores, axis=-1), vf[:, :, None]).reshape(B, Hq, S, D)
        out = out.transpose(0, 2, 1, 3).reshape(B, S, Hq * D)
        return out @ w["wo"].T

    def forward(self, ids, pos):
        """TransformerModel._forward (forward.py:150-159): logits [B, S, V] of
        tokens ids [B, S] at positions pos .. pos+S-1."""
        c = self.cfg
        x = self.w["embed"][ids].astype(np.float32)
        for layer in range(c["num_layers"]):
            w = self.w["layers"][layer]
            h = rms_norm(x, w["n1"], c["norm_eps"])
            x = x + self._attn(layer, h, pos)
            h = rms_norm(x, w["n2"], c["norm_eps"])
            x = x + (silu(h @ w["wg"].T) * (h @ w["wu"].T)) @ w["wd"].T
        x = rms_norm(x, self.w["norm"], c["norm_eps"])
        return x @ self.w["lm_head"].T
