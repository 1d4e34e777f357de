"""GPU: the bounded wait of the NVLink all-reduce gives up and reports it.

A failing peer is made on the host, as a rank that never makes its call: two
comms of one process on one GPU stand for ranks 0 and 1 of world 2 (each rank's
buffer mapped as the other's peer buffer, so every store the kernel makes lands
in valid memory), and only rank 0 launches ``xm_allreduce_add``.  Its wait for
rank 1's flag -- which nothing sets -- runs out after the short limit set on
the comm; the kernel records XM_DEVERR_TIMEOUT in the device error word and
returns, the context stays usable, and the Python layer turns the word into
an exception.  No kernel here waits for another launch.
"""

import ctypes
import time

import pytest
import torch

from xanosmerks_b200 import _lib

pytestmark = pytest.mark.gpu


def _comms(world=2, max_elems=4096, ctas=4):
    lib = _lib.lib
    comms = []
    for r in range(world):
        c = ctypes.c_void_p()
        h = (ctypes.c_ubyte * 64)()
        _lib.check(lib.xm_comm_create(world, r, max_elems, ctas, ctypes.byref(c), h), "comm_create")
        comms.append(c)
    for r in range(world):
        for p in range(world):
            _lib.check(lib.xm_comm_open_local(comms[r], p, comms[p]), "comm_open_local")
    return comms


def test_allreduce_wait_runs_out_when_a_rank_never_arrives():
    lib = _lib.lib
    torch.cuda.set_device(0)
    assert lib.xm_device_status(1) >= 0                  # start from a clear word
    comms = _comms()
    try:
        _lib.check(lib.xm_comm_set_wait_limit(comms[0], 50_000_000), "set_wait_limit")   # 50 ms
        h = torch.zeros(4096, dtype=torch.float32, device="cuda")
        part = torch.ones(4096, dtype=torch.float32, device="cuda")
        st = torch.cuda.current_stream().cuda_stream
        t0 = time.perf_counter()
        _lib.check(lib.xm_allreduce_add(comms[0], h.data_ptr(), part.data_ptr(), 4096, st), "allreduce_add")
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        assert dt < 5.0, dt                              # the limit, not the 2 s default or a hang
        assert lib.xm_device_status(0) & 1 == 1          # XM_DEVERR_TIMEOUT
        with pytest.raises(_lib.XMError):
            _lib.check_device("allreduce")               # raises and clears the word
        assert lib.xm_device_status(0) == 0
        # the context is still usable
        x = torch.arange(8, device="cuda", dtype=torch.float32)
        assert float(x.sum()) == 28.0
    finally:
        torch.cuda.synchronize()
        for c in comms:
            lib.xm_comm_destroy(c)


def test_comm_argument_checks():
    lib = _lib.lib
    comms = _comms()
    try:
        assert lib.xm_comm_set_wait_limit(comms[0], 10) == _lib.XM_ERR_INVALID
        assert lib.xm_comm_open_local(comms[0], 1, comms[0]) == _lib.XM_ERR_INVALID   # rank mismatch
        assert lib.xm_allreduce_add(comms[0], None, None, 4, None) == _lib.XM_ERR_INVALID
    finally:
        for c in comms:
            lib.xm_comm_destroy(c)
