"""A bounded exchange wait that runs out, on one GPU: the counters of an exchange point that
no peer ever publishes (zeros), a short spin limit (2^14 spins, a few ms).  The wait gives up
instead of spinning on, reports 0 to the caller, leaves 0x91 in the device error word, and
the context stays usable: a later wait whose counters are set succeeds and a matvec runs.
Failure is made on the host side (a counter nobody sets); nothing traps or faults."""
import ctypes

import numpy as np
import pytest

from soso_b200 import synth
from soso_b200._lib import lib
from soso_b200.formats import DTYPE_Q4_K

pytestmark = pytest.mark.gpu


def test_exchange_wait_runs_out_and_reports():
    import torch
    L = lib()
    s = torch.cuda.current_stream().cuda_stream
    code = ctypes.c_uint32()
    L.sbk_take_device_error(0, ctypes.byref(code))  # start clean
    cnt = torch.zeros(8, dtype=torch.int32, device="cuda")
    ok = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    assert L.sbk_exchange_wait(cnt.data_ptr(), 2, 1, 1 << 14, ok.data_ptr(), s) == 0
    torch.cuda.synchronize()
    assert int(ok.item()) == 0
    assert L.sbk_take_device_error(0, ctypes.byref(code)) == 0 and code.value == 0x91
    # the context still works: a satisfied wait, then a matvec
    cnt[:2] = 3
    assert L.sbk_exchange_wait(cnt.data_ptr(), 2, 3, 1 << 14, ok.data_ptr(), s) == 0
    torch.cuda.synchronize()
    assert int(ok.item()) == 1
    assert L.sbk_take_device_error(0, ctypes.byref(code)) == 0 and code.value == 0
    g = synth.rng("timeout_mv")
    w = torch.from_numpy(synth.random_weights(DTYPE_Q4_K, 256, 512, g)).cuda()
    x = torch.from_numpy(synth.randn(512, g)).cuda()
    y = torch.full((256,), float("nan"), device="cuda")
    assert L.sbk_matvec(DTYPE_Q4_K, w.data_ptr(), 256, 512, x.data_ptr(), y.data_ptr(), 0, s) == 0
    torch.cuda.synchronize()
    assert np.isfinite(y.cpu().numpy()).all()


def test_exchange_wait_rejects_bad_limits():
    L = lib()
    p = ctypes.c_void_p(256)
    assert L.sbk_exchange_wait(p, 2, 1, 0, p, None) == -1
    assert L.sbk_exchange_wait(p, 9, 1, 100, p, None) == -1
    assert L.sbk_exchange_wait(p, 2, 1, (1 << 26) + 1, p, None) == -1
