"""GPU: the allocation-free decode GEMV agrees with the workspace entry point.

xm_qgemv_noalloc exists for callers that cannot allocate device memory -- for
example a host runtime that owns the device allocator and only lends this
library the tensors it already has.  It keeps the activation split in a fixed
array built into the library instead of a caller-supplied workspace.  This
file sorts last so that a run stopping at its first failure has already run
every other test; it needs no state from them either.
"""

import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import GEMV_TOL, rel_err
from xanosmerks_b200 import _lib
from xanosmerks_b200.synth import make_weight

pytestmark = pytest.mark.gpu

Q4_K = 12


def _with_workspace(w, n, k, x, m, y):
    lib = _lib.lib
    wsz = lib.xm_qgemv_workspace_size(k, m)
    ws = torch.empty(wsz, dtype=torch.uint8, device="cuda")
    _lib.check(lib.xm_qgemv(Q4_K, w.data_ptr(), w.numel(), n, k, x.data_ptr(), _lib.DT_BF16, m, None,
                            y.data_ptr(), ws.data_ptr(), wsz, torch.cuda.current_stream().cuda_stream), "qgemv")


def _no_alloc(w, n, k, x, m, y):
    _lib.check(_lib.lib.xm_qgemv_noalloc(Q4_K, w.data_ptr(), w.numel(), n, k, x.data_ptr(), _lib.DT_BF16, m,
                                         None, y.data_ptr(), torch.cuda.current_stream().cuda_stream),
               "qgemv_noalloc")


@pytest.mark.parametrize("n,k,m", [(11008, 4096, 1), (4096, 14336, 2), (1000, 4096, 8)])
def test_no_alloc_matches_workspace_entry_on_two_calls(n, k, m):
    w = torch.from_numpy(make_weight("Q4_K", n, k, seed=21)).cuda()
    gen = torch.Generator().manual_seed(22)
    for call in range(2):                      # two calls in a row reuse the built-in scratch
        x = torch.randn(m, k, generator=gen).to(torch.bfloat16).cuda()
        y_ref = torch.empty(m, n, dtype=torch.float32, device="cuda")
        y_na = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        _with_workspace(w, n, k, x, m, y_ref)
        _no_alloc(w, n, k, x, m, y_na)
        torch.cuda.synchronize()
        a, b = y_na.cpu().numpy(), y_ref.cpu().numpy()
        assert np.isfinite(a).all(), f"call {call}: output not fully written"
        assert rel_err(a, b) < GEMV_TOL, f"call {call}: {rel_err(a, b)}"


def test_no_alloc_rejects_requests_beyond_the_built_in_scratch():
    lib = _lib.lib
    st = lib.xm_qgemv_noalloc(Q4_K, None, 1 << 40, 16, 32768, None, _lib.DT_BF16, 8, None, None, None)
    assert st == _lib.XM_ERR_INVALID
    assert b"built-in array" in lib.xm_last_error()
