"""Failure detection without a GPU fault: a device-side wait that runs out
returns, records its code in the device status word and leaves the context
usable (the bounded waits every kernel of the library uses).

A one-thread wait kernel polls a device counter that nothing increments,
under a 10 ms wait limit; u15c_sync reports U15C_EDEVICE with the
tensor-parallel wait's code (0x106), u15c_device_status reads it, and a
normal kernel runs correctly afterwards. The limit is restored to its
default before the test ends."""
import ctypes as C

import pytest

from gpu_util import torch

pytestmark = pytest.mark.gpu
WAIT_PEER = 0x106


def test_wait_runs_out_and_reports():
    from u15b200 import _lib as L
    lib = L.lib()
    assert lib.u15c_init(0, 0) == 0
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    counter = torch.zeros(1, dtype=torch.int64, device="cuda")
    code = C.c_uint(0)
    assert lib.u15c_device_status(0, C.byref(code)) == 0   # start clean
    assert lib.u15c_set_wait_limit(0, 10_000_000) == 0      # 10 ms
    try:
        # a counter already at its target passes without a wait
        counter.fill_(3)
        assert lib.u15c_wait_counter(st, C.c_void_p(counter.data_ptr()), 3) == 0
        assert lib.u15c_sync(st) == 0
        # nothing will reach 4: the wait gives up after 10 ms
        assert lib.u15c_wait_counter(st, C.c_void_p(counter.data_ptr()), 4) == 0
        assert lib.u15c_sync(st) == L.EDEVICE
        assert "0x106" in L.last_error()
        # again, read through the status word this time (reading clears it)
        assert lib.u15c_wait_counter(st, C.c_void_p(counter.data_ptr()), 4) == 0
        torch.cuda.synchronize()
        assert lib.u15c_device_status(0, C.byref(code)) == 0
        assert code.value == WAIT_PEER
        assert lib.u15c_device_status(0, C.byref(code)) == 0 and code.value == 0
    finally:
        assert lib.u15c_set_wait_limit(0, 0) == 0
    # the context is intact: a GEMM still runs and matches torch
    a = torch.randn(256, 512, device="cuda").bfloat16()
    w = torch.randn(384, 512, device="cuda").bfloat16()
    y = torch.empty(256, 384, device="cuda").bfloat16()
    assert lib.u15c_linear_bf16(st, C.c_void_p(a.data_ptr()), C.c_void_p(w.data_ptr()), None,
                                C.c_void_p(y.data_ptr()), 256, 512, 384) == 0
    assert lib.u15c_sync(st) == 0
    ref = a.float() @ w.float().t()
    assert ((y.float() - ref).norm() / ref.norm()).item() < 4e-3
