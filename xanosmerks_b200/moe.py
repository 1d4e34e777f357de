"""GPU drop-in for the reference's ``MoELayer`` (moe.py:7-119) on quantized experts.

``MoELayer(config, weights)(x)`` takes the reference's config keys
(``num_experts``, ``num_experts_per_tok``, ``hidden_act``) and its nested
weight dict (``weights["gate"]["weight"]`` -- fp32 router, (E, H) --
and ``weights["experts"][str(i)]["w1" | "w2" | "w3"]["weight"]``), with the
expert weights given as :class:`~xanosmerks_b200.ops.GGUFTensor` (blocks
resident on the GPU).  The same argument checks and exceptions as the
reference are raised.  The forward pass runs entirely on the GPU
(``xm_moe_forward``): routing, stable sort by expert, grouped tensor-core
GEMMs, the gated activation (``hidden_act``: silu/swish, gelu, relu or
identity, as the reference's ``apply_activation``) and the ordered combine.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from ._lib import ACT, DT_BF16, DT_F16, DT_F32, XMError, check, lib
from .ops import GGUFTensor, _workspace

_DT = {torch.float32: DT_F32, torch.bfloat16: DT_BF16, torch.float16: DT_F16}


class MoELayer:
    """Sparse (top-k) or dense (k == E) mixture of gated experts, act(x W1.T) * (x W3.T) then W2
    (act: the reference's ``hidden_act``, silu by default)."""

    def __init__(self, config, weights):
        self.num_experts = config["num_experts"]
        self.num_experts_per_tok = config["num_experts_per_tok"]
        self.activation = config.get("hidden_act", "silu")
        if self.num_experts_per_tok < 1:
            raise ValueError(f"MoELayer: num_experts_per_tok={self.num_experts_per_tok} < 1")
        if self.num_experts_per_tok > self.num_experts:
            raise ValueError(f"MoELayer: num_experts_per_tok={self.num_experts_per_tok} "
                             f"> num_experts={self.num_experts}")
        if self.activation not in ACT:
            raise ValueError(f"MoELayer: unknown activation {self.activation!r} (apply_activation knows "
                             f"{sorted(ACT)})")
        gate_w = weights["gate"]["weight"]
        gate_w = gate_w if isinstance(gate_w, torch.Tensor) else torch.as_tensor(np.asarray(gate_w, np.float32))
        if gate_w.ndim != 2:
            raise ValueError(f"MoELayer: gate.weight must be 2-D, got {gate_w.ndim}-D")
        self.w1, self.w2, self.w3 = [], [], []
        for i in range(self.num_experts):
            exp = weights["experts"][str(i)]
            for name, dst in (("w1", self.w1), ("w2", self.w2), ("w3", self.w3)):
                w = exp[name]["weight"]
                if not isinstance(w, GGUFTensor):
                    raise TypeError("expert weights must be GGUFTensor (quantized blocks resident on the GPU)")
                dst.append(w)
        self.device = self.w1[0].device
        self.gate = gate_w.to(device=self.device, dtype=torch.float32).contiguous()
        self.hidden = self.gate.shape[1]
        self.intermediate = self.w1[0].shape[0]
        qt = {w.qtype.type_id for w in self.w1 + self.w2 + self.w3}
        if len(qt) != 1:
            raise NotImplementedError("all expert weights must share one block type")
        self.qtype = qt.pop()
        E = self.num_experts
        self._p1 = (ctypes.c_void_p * E)(*[w.data.data_ptr() for w in self.w1])
        self._p3 = (ctypes.c_void_p * E)(*[w.data.data_ptr() for w in self.w3])
        self._p2 = (ctypes.c_void_p * E)(*[w.data.data_ptr() for w in self.w2])
        self._is_dense = self.num_experts_per_tok == self.num_experts

    def forward_device(self, x: torch.Tensor) -> torch.Tensor:
        """x: CUDA tensor (..., H) -> fp32 CUDA tensor of the same shape."""
        H, F, E, k = self.hidden, self.intermediate, self.num_experts, self.num_experts_per_tok
        if x.shape[-1] != H:
            raise ValueError(f"x has {x.shape[-1]} features, the router expects {H}")
        if x.dtype not in _DT:
            x = x.float()
        xf = x.reshape(-1, H).contiguous()
        T = xf.shape[0]
        out = torch.empty((T, H), dtype=torch.float32, device=x.device)
        wsz = lib.xm_moe_workspace_size(T, H, F, E, k)
        with torch.cuda.device(x.device):
            stream = torch.cuda.current_stream(x.device)
            ws = _workspace(x.device, stream, wsz)
            check(lib.xm_moe_forward(xf.data_ptr(), _DT[xf.dtype], T, H, self.gate.data_ptr(), E, k, F,
                                     self._p1, self._p3, self._p2, self.qtype, ACT[self.activation], out.data_ptr(),
                                     ws.data_ptr(), ws.numel(), stream.cuda_stream), "moe")
        return out.reshape(x.shape)

    def __call__(self, x):
        """x: (batch, seq, hidden) -> (batch, seq, hidden), as moe.py:54-115.  A numpy x gives a
        numpy fp32 result (the device error word is checked once the result is on the host)."""
        if isinstance(x, torch.Tensor) and x.is_cuda:
            return self.forward_device(x)
        numpy_in = not isinstance(x, torch.Tensor)
        xt = torch.from_numpy(np.ascontiguousarray(np.asarray(x, dtype=np.float32))) if numpy_in else x
        y = self.forward_device(xt.to(self.device))
        with torch.cuda.device(self.device):
            res = y.cpu()
            st = lib.xm_device_status(1)
        if st:
            raise XMError(f"MoELayer: a bounded wait inside a kernel gave up (device error word {st})")
        return res.numpy() if numpy_in else res

    def __repr__(self):
        mode = "dense" if self._is_dense else f"top-{self.num_experts_per_tok}"
        return f"<MoELayer experts={self.num_experts} {mode} activation={self.activation}>"


class MoELayerEP:
    """Expert-parallel MoE block: ``world`` ranks (one process per GPU) each
    hold E / world experts (rank r owns experts r*E/world .. (r+1)*E/world - 1)
    and route their own tokens.  ``forward_device(x)`` on every rank: route and
    sort the local tokens (``xm_moe_dispatch``), exchange the per-expert counts
    and then the selected rows with ``all_to_all`` over the process group
    (NCCL), run the local experts on the received rows as (source rank, local
    expert) groups of the tensor-core grouped GEMM (``xm_moe_experts``),
    exchange the result rows back and combine them in ascending expert order
    (``xm_moe_combine``).  The result equals the single-GPU ``MoELayer`` on the
    same weights.  ``weights`` is the reference's nested dict; only the local
    experts' entries are read."""

    def __init__(self, config, weights, rank: int, world: int, process_group=None):
        import torch.distributed as dist
        self.num_experts = E = config["num_experts"]
        self.num_experts_per_tok = k = config["num_experts_per_tok"]
        if k < 1 or k > E:
            raise ValueError(f"MoELayerEP: num_experts_per_tok={k} outside 1..{E}")
        if E % world:
            raise ValueError(f"MoELayerEP: {E} experts do not divide over {world} ranks")
        self.activation = config.get("hidden_act", "silu")
        if self.activation not in ACT:
            raise ValueError(f"MoELayerEP: unknown activation {self.activation!r}")
        self.rank, self.world = rank, world
        self.pg = process_group if process_group is not None else dist.group.WORLD
        self.e_local = E // world
        gate_w = weights["gate"]["weight"]
        gate_w = gate_w if isinstance(gate_w, torch.Tensor) else torch.as_tensor(np.asarray(gate_w, np.float32))
        self.w1, self.w2, self.w3 = [], [], []
        for i in range(rank * self.e_local, (rank + 1) * self.e_local):
            exp = weights["experts"][str(i)]
            for name, dst in (("w1", self.w1), ("w2", self.w2), ("w3", self.w3)):
                w = exp[name]["weight"]
                if not isinstance(w, GGUFTensor):
                    raise TypeError("expert weights must be GGUFTensor (quantized blocks resident on the GPU)")
                dst.append(w)
        self.device = self.w1[0].device
        self.gate = gate_w.to(device=self.device, dtype=torch.float32).contiguous()
        self.hidden = self.gate.shape[1]
        self.intermediate = self.w1[0].shape[0]
        self.qtype = self.w1[0].qtype.type_id
        # group g = (source rank s, local expert e) -> expert e's weights
        G = world * self.e_local
        self._p1 = (ctypes.c_void_p * G)(*[self.w1[g % self.e_local].data.data_ptr() for g in range(G)])
        self._p3 = (ctypes.c_void_p * G)(*[self.w3[g % self.e_local].data.data_ptr() for g in range(G)])
        self._p2 = (ctypes.c_void_p * G)(*[self.w2[g % self.e_local].data.data_ptr() for g in range(G)])

    def forward_device(self, x: torch.Tensor) -> torch.Tensor:
        """x: this rank's tokens, CUDA (..., H) -> fp32 CUDA tensor of the same shape."""
        H, F, E, k = self.hidden, self.intermediate, self.num_experts, self.num_experts_per_tok
        W, El = self.world, self.e_local
        if x.shape[-1] != H:
            raise ValueError(f"x has {x.shape[-1]} features, the router expects {H}")
        if x.dtype not in _DT:
            x = x.float()
        xf = x.reshape(-1, H).contiguous()
        T = xf.shape[0]
        dev = x.device
        stream = torch.cuda.current_stream(dev)
        st = stream.cuda_stream
        ws = _workspace(dev, stream, lib.xm_moe_workspace_size(T, H, F, E, k))
        send = torch.empty((T * k, H), dtype=xf.dtype, device=dev)
        cnt = torch.empty(E, dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            check(lib.xm_moe_dispatch(xf.data_ptr(), _DT[xf.dtype], T, H, self.gate.data_ptr(), E, k, F,
                                      send.data_ptr(), cnt.data_ptr(), ws.data_ptr(), ws.numel(), st), "moe_dispatch")
            keep = []                                  # device temporaries the experts kernel reads

            def run_experts(recv, rc, off):
                R = recv.shape[0]
                rows = torch.empty((R, H), dtype=torch.float32, device=dev)
                if R:
                    g_cnt = rc.to(dev)
                    g_off = off.to(torch.int32).to(dev)
                    ews = torch.empty(lib.xm_moe_experts_workspace_size(R, H, F), dtype=torch.uint8, device=dev)
                    keep.extend((g_cnt, g_off, ews))
                    check(lib.xm_moe_experts(recv.data_ptr(), _DT[xf.dtype], R, H, F, W * El, g_cnt.data_ptr(),
                                             g_off.data_ptr(), self._p1, self._p3, self._p2, self.qtype,
                                             ACT[self.activation], int(rc.max()), rows.data_ptr(), ews.data_ptr(),
                                             ews.numel(), st),
                          "moe_experts")
                return rows

            back = ep_exchange(send, cnt, W, El, self.pg, run_experts)
            out = torch.empty((T, H), dtype=torch.float32, device=dev)
            check(lib.xm_moe_combine(back.data_ptr(), T, H, E, k, F, ws.data_ptr(), out.data_ptr(), st),
                  "moe_combine")
        return out.reshape(x.shape)


def ep_exchange(send, cnt, world: int, e_local: int, group, run_experts):
    """The host side of expert parallelism between the dispatch and the combine.

    ``send``: this rank's routed rows in ascending expert order (expert e on
    rank e // e_local), ``cnt``: int32 rows per expert.  Exchanges the counts
    and the rows (``all_to_all_single``), calls ``run_experts(recv, rc, off)``
    on the received rows, which arrive grouped by (source rank, local expert)
    with counts ``rc`` and offsets ``off`` (host int tensors), and sends the
    fp32 result rows back; returns them in ``send``'s order.  The tensors may
    live on the GPU (NCCL) or the CPU (gloo)."""
    import torch.distributed as dist
    recv_cnt = torch.empty_like(cnt)                       # [source rank][local expert]
    dist.all_to_all_single(recv_cnt, cnt, group=group)
    c_send = cnt.view(world, e_local).sum(1).cpu().tolist()
    rc = recv_cnt.cpu()
    c_recv = rc.view(world, e_local).sum(1).tolist()
    recv = send.new_empty((int(sum(c_recv)), send.shape[1]))
    dist.all_to_all_single(recv, send, c_recv, c_send, group=group)
    off = torch.cumsum(rc, 0) - rc
    rows = run_experts(recv, rc, off)
    back = rows.new_empty((send.shape[0], rows.shape[1]))
    dist.all_to_all_single(back, rows, c_send, c_recv, group=group)
    return back


__all__ = ["MoELayer", "MoELayerEP", "ep_exchange"]
