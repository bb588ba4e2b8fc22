"""Bounded device-side waits that run out: the time-out path end to end.

The look-back and mbarrier waits of the scan kernels are bounded; a wait that
runs out records MGS_LOOKBACK_TIMEOUT in the call's error word and in the
library's sticky word, and the launch completes. These tests make a wait run
out on purpose through the C ABI's test hooks, with a small poll bound and a
flag or barrier that nothing sets (no planted hang: every wait involved is
bounded), then check that the launch finished, that both error words carry
the bit, that ``take_device_error`` reports and clears it, and that the
context still runs a normal scan correctly afterwards."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TIMEOUT_BIT = 1 << 6  # MGS_LOOKBACK_TIMEOUT


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _scan_still_correct(dev):
    import mingru_b200 as mb
    from oracle import oracle

    g = torch.Generator().manual_seed(7)
    a = torch.tanh(torch.randn(2, 300, 64, generator=g, dtype=torch.float64))
    b = torch.randn(2, 300, 64, generator=g, dtype=torch.float64)
    A, Bc = mb.linear_scan(a.float().to(dev), b.float().to(dev))
    assert mb.take_device_error(dev) == 0
    rA, rB = oracle.linear_scan(a.numpy(), b.numpy())
    np.testing.assert_allclose(A.double().cpu().numpy(), rA, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(Bc.double().cpu().numpy(), rB, rtol=1e-5, atol=1e-6)


def test_lookback_wait_times_out(cuda):
    import mingru_b200 as mb
    from mingru_b200 import _lib

    lib = _lib.load()
    mb.take_device_error(cuda)  # start from a clean sticky word
    Bn, T, D = 2, 512, 64  # 4 strips of 32 lanes: the look-back path, 8 tiles per strip
    a = torch.tanh(torch.randn(Bn, T, D, device=cuda))
    b = torch.randn(Bn, T, D, device=cuda)
    A, Bc = torch.empty_like(a), torch.empty_like(b)
    ws = torch.zeros(max(256, lib.mgs_linear_scan_workspace_size(Bn, T, D, 0)),
                     dtype=torch.uint8, device=cuda)
    st = lib.mgs_test_lookback_timeout(a.data_ptr(), b.data_ptr(), A.data_ptr(), Bc.data_ptr(),
                                       Bn, T, D, ws.data_ptr(), ws.numel(), 256, _stream())
    assert st == 0, _lib.STATUS_NAMES.get(st, st)
    torch.cuda.synchronize()  # the launch completed
    call_err = int(ws[4:8].view(torch.int32).item())
    assert call_err & TIMEOUT_BIT
    assert mb.take_device_error(cuda) & TIMEOUT_BIT
    assert mb.take_device_error(cuda) == 0  # read and cleared
    with pytest.raises(RuntimeError, match="MGS_LOOKBACK_TIMEOUT"):
        lib.mgs_test_lookback_timeout(a.data_ptr(), b.data_ptr(), A.data_ptr(), Bc.data_ptr(),
                                      Bn, T, D, ws.data_ptr(), ws.numel(), 256, _stream())
        mb.raise_device_error(cuda)
    _scan_still_correct(cuda)


def test_lookback_hook_rejects_strip_shapes(cuda):
    from mingru_b200 import _lib

    lib = _lib.load()
    x = torch.empty(16, device=cuda)
    ws = torch.empty(256, dtype=torch.uint8, device=cuda)
    st = lib.mgs_test_lookback_timeout(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                       16, 4096, 1024, ws.data_ptr(), ws.numel(), 256, _stream())
    assert _lib.STATUS_NAMES[st] == "MGS_UNSUPPORTED"


def test_mbarrier_wait_times_out(cuda):
    import mingru_b200 as mb
    from mingru_b200 import _lib

    lib = _lib.load()
    mb.take_device_error(cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    st = lib.mgs_test_mbarrier_timeout(err.data_ptr(), 1000, _stream())
    assert st == 0, _lib.STATUS_NAMES.get(st, st)
    torch.cuda.synchronize()
    assert int(err.item()) & TIMEOUT_BIT
    assert mb.take_device_error(cuda) & TIMEOUT_BIT
    _scan_still_correct(cuda)
