"""GPU: the allocation-free decode GEMV agrees with the workspace entry point.

xm_qgemv_noalloc exists for callers that cannot allocate device memory -- for
example a host runtime that owns the device allocator and only lends this
library the tensors it already has.  It keeps the activation split in a fixed
array built into the library instead of a caller-supplied workspace.  It runs
the same kernels as xm_qgemv with a workspace, so the two results must be
identical bit for bit; both are also checked against the oracle's fp32
``x @ W.T`` on the reference's fp16 weights.  The shapes cover every kernel
family that reads the split from the array (the per-type integer-dot GEMV,
the Q4_K TMA GEMV, the tensor-core GEMV for several rows) up to the array's
limit (8 rows of 16384), plus the single-row K = 4096 Q4_K kernel, which
splits inside its own launch.  This file sorts last so that a run stopping at
its first failure has already run every other test; it needs no state from
them either.
"""

import numpy as np
import pytest
import torch

from oracle import gguf_dequant_oracle as O
from tests.helpers import GEMV_TOL, rel_err
from xanosmerks_b200 import _lib
from xanosmerks_b200.qtypes import normalize
from xanosmerks_b200.synth import make_weight

pytestmark = pytest.mark.gpu


def _with_workspace(qid, w, n, k, x, m, y):
    lib = _lib.lib
    wsz = lib.xm_qgemv_workspace_size(k, m)
    ws = torch.empty(wsz, dtype=torch.uint8, device="cuda")
    _lib.check(lib.xm_qgemv(qid, w.data_ptr(), w.numel(), n, k, x.data_ptr(), _lib.DT_BF16, m, None,
                            y.data_ptr(), ws.data_ptr(), wsz, torch.cuda.current_stream().cuda_stream), "qgemv")
    return ws


def _no_alloc(qid, w, n, k, x, m, y):
    _lib.check(_lib.lib.xm_qgemv_noalloc(qid, w.data_ptr(), w.numel(), n, k, x.data_ptr(), _lib.DT_BF16, m,
                                         None, y.data_ptr(), torch.cuda.current_stream().cuda_stream),
               "qgemv_noalloc")


@pytest.mark.parametrize("name,n,k,m", [
    ("Q4_K", 11008, 4096, 1),    # single-row K = 4096 kernel (split inside the launch)
    ("Q4_K", 4096, 14336, 1),    # Q4_K TMA GEMV from the split
    ("Q6_K", 4096, 4096, 1),     # integer-dot GEMV, digits in registers
    ("Q6_K", 1024, 14336, 1),
    ("Q8_0", 4096, 4096, 1),
    ("Q8_0", 1024, 14336, 1),
    ("Q5_K", 777, 2048, 3),      # several rows: digits in shared memory
    ("Q4_K", 1000, 4096, 8),     # tensor-core GEMV (per-row split)
    ("Q6_K", 512, 16384, 8),     # the array's limit: 8 rows of 16384
])
def test_no_alloc_matches_workspace_entry_on_two_calls(name, n, k, m):
    qid = normalize(name).type_id
    raw = make_weight(name, n, k, seed=21)
    wf = O.dequantize(raw, name, (n, k)).astype(np.float32)
    w = torch.from_numpy(raw).cuda()
    gen = torch.Generator().manual_seed(22)
    for call in range(2):                      # two calls in a row reuse the built-in scratch
        x = torch.randn(m, k, generator=gen).to(torch.bfloat16).cuda()
        y_ref = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        y_na = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        ws = _with_workspace(qid, w, n, k, x, m, y_ref)
        _no_alloc(qid, w, n, k, x, m, y_na)
        torch.cuda.synchronize()
        del ws
        a, b = y_na.cpu().numpy(), y_ref.cpu().numpy()
        assert np.isfinite(a).all(), f"call {call}: output not fully written"
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), \
            f"call {call}: differs from the workspace entry (max |d| {np.abs(a - b).max()})"
        ref = x.float().cpu().numpy() @ wf.T
        assert rel_err(a, ref) < GEMV_TOL, f"call {call}: {rel_err(a, ref)} against the oracle"


def test_no_alloc_rejects_requests_beyond_the_built_in_scratch():
    lib = _lib.lib
    st = lib.xm_qgemv_noalloc(12, None, 1 << 40, 16, 32768, None, _lib.DT_BF16, 8, None, None, None)
    assert st == _lib.XM_ERR_INVALID
    assert b"built-in array" in lib.xm_last_error()
