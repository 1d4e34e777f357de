"""Llama-style decoder on GGUF weights resident in HBM.

The B200 counterpart of the reference's decode loop: ``TransformerModel`` /
``TransformerLayer`` (forward.py:19-160), ``MultiHeadAttention`` with a KV cache
(attention.py:7-115) and the greedy ``Generator`` step (generate.py,
sampling.py:51-52).  Every projection runs on the quantized blocks through the
C ABI (``xm_qgemv_ex``: the attention RMSNorm is fused into the QKV GEMV, the
MLP RMSNorm into the gate/up GEMV, SwiGLU into the down GEMV, the residual adds
into the O and down GEMVs), plus three small kernels (embedding gather,
attention with RoPE and the KV append fused in, argmax).  A decode step is 5-6
launches per layer and is captured once into a CUDA graph.

Layout: per layer the Q, K, V rows are concatenated into one GGUF tensor (one
GEMV), and so are gate and up; the caches are fp16 ``[B][Hk][max_ctx][128]``.

Tensor parallelism (``world_size > 1``, one process per GPU): attention heads
and FFN columns are split across ranks (QKV and gate/up column-parallel, O and
down row-parallel over K, so each rank holds the K-slice of every row), the two
row-parallel partial sums are all-reduced over NCCL, and the embedding and
output projection are replicated.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import qtypes
from ._lib import DT_F32, PRO_NONE, PRO_RMSNORM, PRO_SWIGLU, check, check_device, lib
from .ops import GGUFTensor, gemm_supported
from .synth import make_weight_device

__all__ = ["LlamaConfig", "LlamaWeights", "LlamaDecoder", "synth_llama_weights", "shard_rows", "shard_cols"]

# |N(0,1)| * scale for the fp16 scale fields gives weights of rms ~0.02 (a
# trained model's magnitude), so activations stay O(1) through the layers
_WEIGHT_SCALE = {"Q4_K": 6.75e-5, "Q6_K": 1.45e-5, "Q5_K": 3.5e-5, "Q8_0": 1.6e-4}


@dataclass
class LlamaConfig:
    num_layers: int = 32
    hidden_size: int = 4096
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 14336
    vocab_size: int = 32000
    norm_eps: float = 1e-5
    rope_theta: float = 5e5
    attn_qtype: str = "Q4_K"
    gate_up_qtype: str = "Q4_K"
    down_qtype: str = "Q6_K"
    output_qtype: str = "Q6_K"
    embed_qtype: str = "Q4_K"

    def reference_config(self) -> dict:
        """The keys the reference's model classes read (forward.py, attention.py)."""
        return {"num_layers": self.num_layers, "hidden_size": self.hidden_size, "num_heads": self.num_heads,
                "num_kv_heads": self.num_kv_heads, "head_dim": self.head_dim,
                "intermediate_size": self.intermediate_size, "vocab_size": self.vocab_size,
                "norm_eps": self.norm_eps, "rope_theta": self.rope_theta, "hidden_act": "silu",
                "norm_type": "rmsnorm"}

    def weight_bytes_per_token(self) -> int:
        """Quantized bytes one decode step streams (all projections incl. the output head)."""
        D, F, V = self.hidden_size, self.intermediate_size, self.vocab_size
        qkv = (self.num_heads + 2 * self.num_kv_heads) * self.head_dim
        rb = lambda q, n, k: n * qtypes.row_bytes(qtypes.normalize(q), k)  # noqa: E731
        layer = (rb(self.attn_qtype, qkv, D) + rb(self.attn_qtype, D, self.num_heads * self.head_dim)
                 + rb(self.gate_up_qtype, 2 * F, D) + rb(self.down_qtype, D, F))
        return self.num_layers * layer + rb(self.output_qtype, V, D)


def _blocks(t: GGUFTensor) -> torch.Tensor:
    """The tensor's bytes as [n rows][blocks per row][record]."""
    q = t.qtype
    n, k = t.shape
    return t.data.view(n, k // q.qk, q.record)


def shard_rows(t: GGUFTensor, r0: int, r1: int) -> GGUFTensor:
    """Rows [r0, r1) (a column-parallel shard: whole rows, contiguous bytes)."""
    n, k = t.shape
    rb = qtypes.row_bytes(t.qtype, k)
    return GGUFTensor(t.data[r0 * rb:r1 * rb], t.qtype.name, (r1 - r0, k))


def shard_cols(t: GGUFTensor, k0: int, k1: int) -> GGUFTensor:
    """Columns [k0, k1) of every row (a row-parallel shard over K), copied to a
    contiguous tensor; k0, k1 must fall on block boundaries."""
    q = t.qtype
    n, k = t.shape
    if k0 % q.qk or k1 % q.qk:
        raise ValueError(f"K-slice [{k0}, {k1}) does not fall on {q.name} block boundaries ({q.qk})")
    part = _blocks(t)[:, k0 // q.qk:k1 // q.qk, :].contiguous().view(-1)
    return GGUFTensor(part, q.name, (n, k1 - k0))


def _cat_rows(parts) -> GGUFTensor:
    q = parts[0].qtype
    k = parts[0].shape[1]
    return GGUFTensor(torch.cat([p.data for p in parts]), q.name, (sum(p.shape[0] for p in parts), k))


class LlamaWeights:
    """One rank's weights.  ``layers[i]``: ``qkv`` [(Hq+2Hk)*128, D] (this rank's
    heads), ``o`` [D, Hq*128 / world], ``gate_up`` [2F / world, D] (gate rows then
    up rows), ``down`` [D, F / world], ``attn_norm`` / ``ffn_norm`` fp32 [D];
    ``embed`` [V, D], ``norm`` fp32 [D], ``output`` [V, D]."""

    def __init__(self, cfg: LlamaConfig, embed, layers, norm, output, rank=0, world=1):
        self.cfg, self.embed, self.layers, self.norm, self.output = cfg, embed, layers, norm, output
        self.rank, self.world = rank, world

    @classmethod
    def from_full(cls, cfg: LlamaConfig, full: dict, rank: int = 0, world: int = 1) -> "LlamaWeights":
        """Shard full per-layer tensors ``wq, wk, wv, wo, wg, wu, wd`` (GGUFTensor)
        and ``n1, n2`` for ``rank`` of ``world``."""
        hq, hk, hd, F = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.intermediate_size
        if hq % world or hk % world or F % world:
            raise ValueError(f"heads {hq}/{hk} and FFN {F} must divide by the world size {world}")
        hq_l, hk_l, f_l = hq // world, hk // world, F // world
        layers = []
        for lw in full["layers"]:
            qkv = _cat_rows([shard_rows(lw["wq"], rank * hq_l * hd, (rank + 1) * hq_l * hd),
                             shard_rows(lw["wk"], rank * hk_l * hd, (rank + 1) * hk_l * hd),
                             shard_rows(lw["wv"], rank * hk_l * hd, (rank + 1) * hk_l * hd)])
            o = lw["wo"] if world == 1 else shard_cols(lw["wo"], rank * hq_l * hd, (rank + 1) * hq_l * hd)
            gu = _cat_rows([shard_rows(lw["wg"], rank * f_l, (rank + 1) * f_l),
                            shard_rows(lw["wu"], rank * f_l, (rank + 1) * f_l)])
            down = lw["wd"] if world == 1 else shard_cols(lw["wd"], rank * f_l, (rank + 1) * f_l)
            layers.append({"qkv": qkv, "o": o, "gate_up": gu, "down": down,
                           "attn_norm": lw["n1"], "ffn_norm": lw["n2"]})
        return cls(cfg, full["embed"], layers, full["norm"], full["output"], rank, world)


def synth_llama_weights(cfg: LlamaConfig, seed: int = 0, device="cuda"):
    """Random-init weights in the config's GGUF types (seeded, generated on the
    device): the full (unsharded) tensors as a dict of GGUFTensor / fp32 norms."""
    device = torch.device(device)
    D, F, V, hd = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.head_dim
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def w(qt, n, k, s):
        raw = make_weight_device(qt, n, k, seed=seed * 100003 + s, device=device, scale=_WEIGHT_SCALE.get(qt))
        return GGUFTensor(raw, qt, (n, k), device=device)

    def norm_w():
        return (1.0 + 0.05 * torch.randn(D, generator=g, device=device)).float()

    layers = []
    for i in range(cfg.num_layers):
        b = 16 * (i + 1)
        layers.append({"wq": w(cfg.attn_qtype, cfg.num_heads * hd, D, b + 0),
                       "wk": w(cfg.attn_qtype, cfg.num_kv_heads * hd, D, b + 1),
                       "wv": w(cfg.attn_qtype, cfg.num_kv_heads * hd, D, b + 2),
                       "wo": w(cfg.attn_qtype, D, cfg.num_heads * hd, b + 3),
                       "wg": w(cfg.gate_up_qtype, F, D, b + 4),
                       "wu": w(cfg.gate_up_qtype, F, D, b + 5),
                       "wd": w(cfg.down_qtype, D, F, b + 6),
                       "n1": norm_w(), "n2": norm_w()})
    return {"embed": w(cfg.embed_qtype, V, D, 1), "layers": layers, "norm": norm_w(),
            "output": w(cfg.output_qtype, V, D, 2)}


class LlamaDecoder:
    """Greedy decoder for ``batch`` sequences of up to ``max_ctx`` tokens.

    ``prefill(ids)`` runs the prompt (ids [B, S]) through the layers, 8 tokens
    per sequence at a time, and returns the next token of each sequence;
    ``decode_step()`` advances every sequence by one token (embedding of the
    last token -> layers -> output head -> argmax), reading and writing only
    device state, so that it can be captured into a CUDA graph
    (``capture()`` / ``replay()``).  ``process_group``: the tensor-parallel group
    when the weights are a shard of ``world > 1``; ``collective`` selects the
    exchange of the row-parallel partial sums: ``"p2p"`` (default: the one-shot
    all-reduce over NVLink peer memory of ``xm_allreduce_add``, buffers shared
    through CUDA IPC) or ``"nccl"`` (``torch.distributed.all_reduce``).  Call
    ``close()`` on every rank before tearing the process group down.
    """

    LQ_MAX = 8
    COMM_CTAS = 16

    def __init__(self, weights: LlamaWeights, batch: int, max_ctx: int, device=None, process_group=None,
                 collective: str = "p2p"):
        cfg = weights.cfg
        self.cfg, self.w, self.B, self.max_ctx = cfg, weights, int(batch), int(max_ctx)
        self.world = weights.world
        self.pg = process_group
        if self.world > 1 and process_group is None:
            import torch.distributed as dist
            self.pg = dist.group.WORLD
        dev = torch.device(device) if device is not None else weights.embed.device
        self.dev = dev
        self.hq = cfg.num_heads // self.world
        self.hk = cfg.num_kv_heads // self.world
        hd, D = cfg.head_dim, cfg.hidden_size
        self.qkv_dim = (self.hq + 2 * self.hk) * hd
        self.f_l = cfg.intermediate_size // self.world
        rows = self.B * self.LQ_MAX
        f32 = dict(dtype=torch.float32, device=dev)
        self.h = torch.zeros(rows, D, **f32)
        self.qkv = torch.zeros(rows, self.qkv_dim, **f32)
        self.attn = torch.zeros(rows, self.hq * hd, **f32)
        self.gu = torch.zeros(rows, 2 * self.f_l, **f32)
        self.part = torch.zeros(rows, D, **f32)          # row-parallel partial sums (world > 1)
        self.logits = torch.zeros(self.B, cfg.vocab_size, **f32)
        i32 = dict(dtype=torch.int32, device=dev)
        self.ids = torch.zeros(rows, **i32)               # token ids of the rows being processed
        self.next_ids = torch.zeros(self.B, **i32)
        self.pos0 = torch.zeros(self.B, **i32)            # tokens already in the cache per sequence
        self.kc = torch.zeros(cfg.num_layers, self.B, self.hk, self.max_ctx, hd, dtype=torch.float16, device=dev)
        self.vc = torch.zeros_like(self.kc)
        aws = lib.xm_attention_workspace_size(self.B, self.hk, self.max_ctx)
        self.attn_ws = torch.zeros(aws, dtype=torch.uint8, device=dev)
        kmax = max(D, cfg.intermediate_size, self.hq * hd)
        self.gemv_ws = torch.zeros(lib.xm_qgemv_workspace_size(kmax, 8) + 4096, dtype=torch.uint8, device=dev)
        self.graph = None
        self.length = 0
        self.comm = None
        self._gemm_ws = None
        # decode-step GEMMs (4+ rows) get a workspace of their own, allocated once: a captured step
        # keeps its pointer, and the prefill's workspace may be replaced when a longer prompt comes
        dec_need = 16
        for wt in list(self.w.layers[0].values()) + [self.w.output]:
            if isinstance(wt, GGUFTensor) and len(wt.shape) == 2:
                r = self.B if wt is self.w.output else rows
                dec_need = max(dec_need, lib.xm_qgemm_workspace_size_n(r, wt.shape[0], wt.shape[1]))
        self.dec_gemm_ws = torch.zeros(dec_need, dtype=torch.uint8, device=dev)
        # K-slices whose rows are not whole 16-byte units (tensor-parallel Q6_K down projections: 7168
        # columns are 5880 bytes a row) keep a copy with each row padded to a 16-byte pitch for the
        # GEMM (prefill and 4+-row steps); the GEMV reads the packed slice
        self._pitched = {}
        for lw in self.w.layers:
            for wt in lw.values():
                if not (isinstance(wt, GGUFTensor) and len(wt.shape) == 2):
                    continue
                n, k = wt.shape
                rb = qtypes.row_bytes(wt.qtype, k)
                if k % 256 or rb % 16 == 0:
                    continue
                pitch = (rb + 15) // 16 * 16
                pad = torch.zeros(n, pitch, dtype=torch.uint8, device=dev)
                pad[:, :rb] = wt.data.view(n, rb)
                self._pitched[wt.data.data_ptr()] = (pad, pitch)
        if collective not in ("p2p", "nccl"):
            raise ValueError(f"collective must be 'p2p' or 'nccl', got {collective!r}")
        self.collective = collective
        if self.world > 1 and collective == "p2p":
            self._open_comm(rows * D)

    def _open_comm(self, max_elems):
        import ctypes

        import torch.distributed as dist
        rank = self.w.rank
        comm = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        with torch.cuda.device(self.dev):
            check(lib.xm_comm_create(self.world, rank, max_elems, self.COMM_CTAS, ctypes.byref(comm), handle),
                  "comm_create")
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=self.pg)
            for r, hb in enumerate(handles):
                buf = (ctypes.c_ubyte * 64).from_buffer_copy(hb)
                check(lib.xm_comm_open_peer(comm, r, buf), "comm_open_peer")
        self.comm = comm
        dist.barrier(group=self.pg)

    def close(self):
        """Release the CUDA graph and the peer-memory buffers (every rank, after its last step)."""
        self.graph = None
        if self.comm is not None:
            import torch.distributed as dist
            torch.cuda.synchronize(self.dev)
            dist.barrier(group=self.pg)           # no rank still writes into another's buffer
            check(lib.xm_comm_destroy(self.comm), "comm_destroy")
            self.comm = None

    # -- launches ---------------------------------------------------------
    def _stream(self):
        return torch.cuda.current_stream(self.dev).cuda_stream

    def _gemv(self, wt: GGUFTensor, x: torch.Tensor, rows: int, y: torch.Tensor, prologue=PRO_NONE, norm=None,
              accumulate=False):
        """y[:rows] (+)= pro(x[:rows]) @ W.T, in groups of <= 8 rows."""
        n, k = wt.shape
        for r0 in range(0, rows, 8):
            m = min(8, rows - r0)
            check(lib.xm_qgemv_ex(wt.qtype.type_id, wt.data.data_ptr(), wt.nbytes, n, k, x[r0:r0 + m].data_ptr(),
                                  DT_F32, m, x.stride(0), prologue, norm.data_ptr() if norm is not None else None,
                                  self.cfg.norm_eps, None, y[r0:r0 + m].data_ptr(), 1 if accumulate else 0,
                                  self.gemv_ws.data_ptr(), self.gemv_ws.numel(), self._stream()), "qgemv_ex")

    def _allreduce_add(self, rows):
        """h[:rows] += sum over ranks of part[:rows] (row-parallel outputs)."""
        if self.comm is not None:
            n = rows * self.cfg.hidden_size
            check(lib.xm_allreduce_add(self.comm, self.h.data_ptr(), self.part.data_ptr(), n, self._stream()),
                  "allreduce_add")
            return
        import torch.distributed as dist
        p = self.part[:rows]
        dist.all_reduce(p, group=self.pg)
        self.h[:rows].add_(p)

    def _layers(self, lq: int):
        cfg, B = self.cfg, self.B
        rows = B * lq
        st = self._stream()
        for li, lw in enumerate(self.w.layers):
            # attention block (forward.py:107-111)
            self._proj(lw["qkv"], self.h, rows, self.qkv, PRO_RMSNORM, lw["attn_norm"])
            check(lib.xm_attention(self.qkv.data_ptr(), self.qkv_dim, self.kc[li].data_ptr(),
                                   self.vc[li].data_ptr(), self.pos0.data_ptr(), B, lq, self.hq, self.hk,
                                   cfg.head_dim, cfg.rope_theta, self.max_ctx, self.attn.data_ptr(),
                                   self.hq * cfg.head_dim, self.attn_ws.data_ptr(), self.attn_ws.numel(), st),
                  "attention")
            if self.world == 1:
                self._proj(lw["o"], self.attn, rows, self.h, accumulate=True)
            else:
                self._proj(lw["o"], self.attn, rows, self.part)
                self._allreduce_add(rows)
            # MLP block (forward.py:113-116)
            self._proj(lw["gate_up"], self.h, rows, self.gu, PRO_RMSNORM, lw["ffn_norm"])
            if self.world == 1:
                self._proj(lw["down"], self.gu, rows, self.h, PRO_SWIGLU, accumulate=True)
            else:
                self._proj(lw["down"], self.gu, rows, self.part, PRO_SWIGLU)
                self._allreduce_add(rows)

    def _head(self, lq: int):
        """Final RMSNorm + output projection of each sequence's last row, then argmax."""
        D = self.cfg.hidden_size
        ow = self.w.output
        if self.B >= self.GEMM_DECODE_ROWS and ow.qtype.name != "Q4_K" and gemm_supported(ow.qtype, ow.shape[1]):
            last = self.h[:self.B * lq].view(self.B, lq, D)[:, lq - 1]     # each sequence's last row
            self._gemm(ow, last, self.B, self.logits, PRO_RMSNORM, self.w.norm, ws=self.dec_gemm_ws)
            check(lib.xm_argmax(self.logits.data_ptr(), self.B, self.cfg.vocab_size, self.next_ids.data_ptr(),
                                self._stream()), "argmax")
            return
        for b0 in range(0, self.B, 8):
            m = min(8, self.B - b0)
            xp = self.h.data_ptr() + ((b0 * lq + lq - 1) * D) * 4
            check(lib.xm_qgemv_ex(ow.qtype.type_id, ow.data.data_ptr(), ow.nbytes, ow.shape[0], ow.shape[1], xp,
                                  DT_F32, m, lq * D, PRO_RMSNORM, self.w.norm.data_ptr(), self.cfg.norm_eps, None,
                                  self.logits[b0:b0 + m].data_ptr(), 0, self.gemv_ws.data_ptr(),
                                  self.gemv_ws.numel(), self._stream()), "output head")
        check(lib.xm_argmax(self.logits.data_ptr(), self.B, self.cfg.vocab_size, self.next_ids.data_ptr(),
                            self._stream()), "argmax")

    def _embed(self, rows, ids):
        e = self.w.embed
        check(lib.xm_embed(e.qtype.type_id, e.data.data_ptr(), e.nbytes, e.shape[0], e.shape[1],
                           ids.data_ptr(), rows, self.h.data_ptr(), self._stream()), "embed")

    # -- public API -------------------------------------------------------
    def reset(self):
        self.pos0.zero_()
        self.length = 0
        self.graph = None

    def forward_tokens(self, ids: torch.Tensor) -> torch.Tensor:
        """Run ids [B, lq] (lq <= 8) at the current positions; returns the next token per sequence."""
        B, lq = ids.shape
        if B != self.B or not 1 <= lq <= self.LQ_MAX:
            raise ValueError(f"ids must be [{self.B}, 1..{self.LQ_MAX}], got {tuple(ids.shape)}")
        if self.length + lq > self.max_ctx:
            raise ValueError(f"context overflow: {self.length} + {lq} > {self.max_ctx}")
        rows = B * lq
        lo, hi = int(ids.min()), int(ids.max())
        if lo < 0 or hi >= self.cfg.vocab_size:
            raise ValueError(f"token ids must lie in [0, {self.cfg.vocab_size}), got [{lo}, {hi}]")
        self.ids[:rows].copy_(ids.reshape(-1).to(self.dev, torch.int32))
        self._embed(rows, self.ids)
        self._layers(lq)
        self._head(lq)
        self.pos0.add_(lq)
        self.length += lq
        return self.next_ids

    def logits_of_last(self) -> torch.Tensor:
        return self.logits

    def prefill(self, ids) -> torch.Tensor:
        """Prompt ids [B, S] -> next token per sequence (the prompt enters the cache).

        A prompt of more than 8 tokens entering an empty cache runs every projection once over all
        B*S rows on the tensor-core GEMM (RMSNorm, SwiGLU and the residual adds fused as in decode)
        and the attention in chunks of up to 64 tokens per sequence; shorter prompts, and prompts
        appended to a filled cache, go 8 tokens at a time through the decode path."""
        ids = torch.as_tensor(np.asarray(ids) if not isinstance(ids, torch.Tensor) else ids)
        B, S = ids.shape
        if S > self.LQ_MAX and self.length == 0:
            return self._prefill_gemm(ids)
        out = None
        for s0 in range(0, S, self.LQ_MAX):
            out = self.forward_tokens(ids[:, s0:s0 + self.LQ_MAX])
        return out

    PREFILL_CHUNK = 64

    def _gemm(self, wt: GGUFTensor, x: torch.Tensor, rows: int, y: torch.Tensor, prologue=PRO_NONE, norm=None,
              accumulate=False, ws=None):
        """y[:rows] (+)= pro(x[:rows]) @ W.T on the tensor-core GEMM (GEMV groups where the type's row
        pitch does not suit the GEMM).  `ws`: a fixed workspace (decode steps), else the prefill's."""
        n, k = wt.shape
        pitched = self._pitched.get(wt.data.data_ptr())
        if not gemm_supported(wt.qtype, k) and pitched is None:
            self._gemv(wt, x, rows, y, prologue, norm, accumulate)
            return
        if ws is None:
            need = lib.xm_qgemm_workspace_size_n(rows, n, k)
            if self._gemm_ws is None or self._gemm_ws.numel() < need:
                self._gemm_ws = torch.empty(need, dtype=torch.uint8, device=self.dev)
            ws = self._gemm_ws
        norm_p = norm.data_ptr() if norm is not None else None
        if pitched is not None:
            pad, pitch = pitched
            check(lib.xm_qgemm_ex_pitched(wt.qtype.type_id, pad.data_ptr(), pitch, pad.numel(), n, k, x.data_ptr(),
                                          DT_F32, rows, x.stride(0), prologue, norm_p, self.cfg.norm_eps, None,
                                          y.data_ptr(), 1 if accumulate else 0, ws.data_ptr(), ws.numel(),
                                          self._stream()), "qgemm_ex_pitched")
            return
        check(lib.xm_qgemm_ex(wt.qtype.type_id, wt.data.data_ptr(), wt.nbytes, n, k, x.data_ptr(), DT_F32, rows,
                              x.stride(0), prologue, norm_p, self.cfg.norm_eps, None, y.data_ptr(),
                              1 if accumulate else 0, ws.data_ptr(), ws.numel(), self._stream()), "qgemm_ex")

    # Decode steps with this many rows or more run the block types whose multi-row GEMV is the
    # integer-dot kernel (every type but Q4_K, which has the tensor-core GEMV) on the tcgen05 GEMM
    # instead: at 4-8 rows the dp4a work per weight grows with the rows, while the GEMM's cost per
    # weight tile is the decode of the tile (Q6_K 4096x14336 at 8 rows: ~40 us against ~100 us).
    GEMM_DECODE_ROWS = 4

    def _proj(self, wt: GGUFTensor, x: torch.Tensor, rows: int, y: torch.Tensor, prologue=PRO_NONE, norm=None,
              accumulate=False):
        """A decode projection: the GEMV, or the GEMM for 4+ rows of a non-Q4_K weight."""
        if rows >= self.GEMM_DECODE_ROWS and wt.qtype.name != "Q4_K" and (
                gemm_supported(wt.qtype, wt.shape[1]) or wt.data.data_ptr() in self._pitched):
            self._gemm(wt, x, rows, y, prologue, norm, accumulate, ws=self.dec_gemm_ws)
        else:
            self._gemv(wt, x, rows, y, prologue, norm, accumulate)

    def _prefill_gemm(self, ids: torch.Tensor) -> torch.Tensor:
        cfg, B = self.cfg, self.B
        S = ids.shape[1]
        if ids.shape[0] != B:
            raise ValueError(f"ids must be [{B}, S], got {tuple(ids.shape)}")
        if S > self.max_ctx:
            raise ValueError(f"context overflow: {S} > {self.max_ctx}")
        lo, hi = int(ids.min()), int(ids.max())
        if lo < 0 or hi >= cfg.vocab_size:
            raise ValueError(f"token ids must lie in [0, {cfg.vocab_size}), got [{lo}, {hi}]")
        rows = B * S                                       # row b*S + s: token s of sequence b
        D, hd = cfg.hidden_size, cfg.head_dim
        f32 = dict(dtype=torch.float32, device=self.dev)
        h = torch.empty(rows, D, **f32)
        qkv = torch.empty(rows, self.qkv_dim, **f32)
        attn = torch.empty(rows, self.hq * hd, **f32)
        gu = torch.empty(rows, 2 * self.f_l, **f32)
        part = torch.empty(rows, D, **f32) if self.world > 1 else None
        idv = ids.reshape(-1).to(self.dev, torch.int32).contiguous()
        chunk_pos = torch.arange(0, S, self.PREFILL_CHUNK, dtype=torch.int32, device=self.dev)
        st = self._stream()
        e = self.w.embed
        check(lib.xm_embed(e.qtype.type_id, e.data.data_ptr(), e.nbytes, e.shape[0], e.shape[1], idv.data_ptr(),
                           rows, h.data_ptr(), st), "embed")
        # 16 or more tokens: one attention call over all sequences (the tensor-core prefill path)
        whole = S >= 16
        zeros_b = torch.zeros(B, dtype=torch.int32, device=self.dev)
        for li, lw in enumerate(self.w.layers):
            self._gemm(lw["qkv"], h, rows, qkv, PRO_RMSNORM, lw["attn_norm"])
            if whole:
                check(lib.xm_attention(qkv.data_ptr(), self.qkv_dim, self.kc[li].data_ptr(), self.vc[li].data_ptr(),
                                       zeros_b.data_ptr(), B, S, self.hq, self.hk, hd, cfg.rope_theta,
                                       self.max_ctx, attn.data_ptr(), self.hq * hd, self.attn_ws.data_ptr(),
                                       self.attn_ws.numel(), st), "attention")
            for b in range(B if not whole else 0):
                for ci, c0 in enumerate(range(0, S, self.PREFILL_CHUNK)):
                    lq = min(self.PREFILL_CHUNK, S - c0)
                    r0 = b * S + c0
                    check(lib.xm_attention(qkv[r0].data_ptr(), self.qkv_dim, self.kc[li, b].data_ptr(),
                                           self.vc[li, b].data_ptr(), chunk_pos[ci].data_ptr(), 1, lq, self.hq,
                                           self.hk, hd, cfg.rope_theta, self.max_ctx, attn[r0].data_ptr(),
                                           self.hq * hd, self.attn_ws.data_ptr(), self.attn_ws.numel(), st),
                          "attention")
            if self.world == 1:
                self._gemm(lw["o"], attn, rows, h, accumulate=True)
            else:
                self._gemm(lw["o"], attn, rows, part)
                self._allreduce_rows(h, part)
            self._gemm(lw["gate_up"], h, rows, gu, PRO_RMSNORM, lw["ffn_norm"])
            if self.world == 1:
                self._gemm(lw["down"], gu, rows, h, PRO_SWIGLU, accumulate=True)
            else:
                self._gemm(lw["down"], gu, rows, part, PRO_SWIGLU)
                self._allreduce_rows(h, part)
        # the output head on each sequence's last token (the decode state keeps those rows)
        last = h.view(B, S, D)[:, S - 1]
        self.h[:B].copy_(last)
        self._head(1)
        self.pos0.fill_(S)
        self.length = S
        return self.next_ids

    def _allreduce_rows(self, h, part):
        """h += sum over ranks of part (the prefill's row-parallel outputs, NCCL all-reduce)."""
        import torch.distributed as dist
        dist.all_reduce(part, group=self.pg)
        h.add_(part)

    def decode_step(self):
        """One greedy step from device state: the token in next_ids enters at pos0."""
        B = self.B
        self._embed(B, self.next_ids)
        self._layers(1)
        self._head(1)
        self.pos0.add_(1)

    def capture(self):
        """Capture decode_step into a CUDA graph (call after a warm-up step)."""
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.decode_step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.graph = g
        return g

    def replay(self, n: int = 1):
        """n graph-captured decode steps (each advances every sequence by one token)."""
        if self.length + n > self.max_ctx:
            raise ValueError("context overflow")
        for _ in range(n):
            self.graph.replay()
        self.length += n

    def check(self):
        """Raise if a bounded wait inside any kernel since the last check gave up (a tensor-parallel
        peer that never arrived, a lost bulk copy); synchronises the device.  ``generate`` calls it
        after every token; callers that drive ``replay`` themselves call it where they read results."""
        with torch.cuda.device(self.dev):
            check_device("LlamaDecoder")

    def generate(self, prompt, max_new_tokens: int, use_graph: bool = True) -> np.ndarray:
        """Greedy generation: prompt [B, S] -> generated ids [B, max_new_tokens]."""
        self.reset()
        out = np.zeros((self.B, max_new_tokens), dtype=np.int64)
        nxt = self.prefill(prompt)
        out[:, 0] = nxt.cpu().numpy()
        self.check()
        for t in range(1, max_new_tokens):
            if use_graph:
                if self.graph is None:
                    self.decode_step()
                    self.length += 1
                    out[:, t] = self.next_ids.cpu().numpy()
                    self.capture()
                    continue
                self.replay(1)
            else:
                self.decode_step()
                self.length += 1
            out[:, t] = self.next_ids.cpu().numpy()
            self.check()
        return out
