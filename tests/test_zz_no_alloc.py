"""The allocation-free linear_scan forward (mgs_linear_scan_fwd_noalloc).

Callers that cannot hand the library a workspace (allocation forbidden or
synchronising where they run) use this entry point; its scratch is a fixed
device array inside the library. This file is collected last on purpose:
the entry point's scratch is shared process-wide, so the check runs after
every other test has used the library in the same process, and also passes
on its own in a fresh process. Tolerance: the fp32 forward tolerance of the
other parity tests (rtol 1e-5 / atol 1e-6) -- in practice both entry points
run the same kernels and agree exactly."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _fwd_reference(lib, a, b, carries):
    """The allocating entry point, with a workspace from torch."""
    Bn, T, D = a.shape
    A, Bc = torch.empty_like(a), torch.empty_like(b)
    ws = torch.empty(max(256, lib.mgs_linear_scan_workspace_size(Bn, T, D, 0)),
                     dtype=torch.uint8, device=a.device)
    st = lib.mgs_linear_scan_fwd(a.data_ptr(), b.data_ptr(), A.data_ptr(), Bc.data_ptr(),
                                 carries.data_ptr() if carries is not None else None,
                                 Bn, T, D, 0, ws.data_ptr(), ws.numel(),
                                 torch.cuda.current_stream().cuda_stream)
    assert st == 0
    return A, Bc


def _fwd_noalloc(lib, a, b, carries):
    Bn, T, D = a.shape
    A, Bc = torch.empty_like(a), torch.empty_like(b)
    st = lib.mgs_linear_scan_fwd_noalloc(a.data_ptr(), b.data_ptr(), A.data_ptr(), Bc.data_ptr(),
                                         carries.data_ptr() if carries is not None else None,
                                         Bn, T, D, 0, torch.cuda.current_stream().cuda_stream)
    return st, A, Bc


@pytest.mark.parametrize("shape", [(2, 300, 256), (3, 1000, 37), (16, 4096, 1024), (1, 33, 8)])
def test_noalloc_matches_allocating_entry_point(cuda, shape):
    from mingru_b200 import _lib

    lib = _lib.load()
    g = torch.Generator(device=cuda).manual_seed(sum(shape))
    for call in range(2):  # two calls in a row share (and must re-clear) the scratch
        a = torch.tanh(torch.randn(shape, device=cuda, generator=g))
        b = torch.randn(shape, device=cuda, generator=g)
        csz = lib.mgs_linear_scan_carry_size(*shape, 0) // 4
        car_ref = torch.empty(csz, device=cuda)
        car_na = torch.empty(csz, device=cuda)
        A_ref, B_ref = _fwd_reference(lib, a, b, car_ref)
        st, A_na, B_na = _fwd_noalloc(lib, a, b, car_na)
        assert st == 0, _lib.STATUS_NAMES.get(st, st)
        torch.cuda.synchronize()
        assert lib.mgs_take_device_error(torch.cuda.current_stream().cuda_stream) == 0
        torch.testing.assert_close(A_na, A_ref, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(B_na, B_ref, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(car_na, car_ref, rtol=1e-5, atol=1e-6)
        if a.numel() <= 1 << 20:  # and directly against the fp64 oracle
            from oracle import oracle

            rA, rB = oracle.linear_scan(a.double().cpu().numpy(), b.double().cpu().numpy())
            np.testing.assert_allclose(A_na.double().cpu().numpy(), rA, rtol=1e-5, atol=1e-6)
            np.testing.assert_allclose(B_na.double().cpu().numpy(), rB, rtol=1e-5, atol=1e-6)


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    from mingru_b200 import _lib

    lib = _lib.load()
    # a narrow (look-back) shape whose scratch needs more than the fixed array
    Bn, T, D = 1, 1 << 22, 256
    need = lib.mgs_linear_scan_workspace_size(Bn, T, D, 0)
    assert need > 32 << 20
    x = torch.empty(1, device=cuda)
    st = lib.mgs_linear_scan_fwd_noalloc(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                         None, Bn, T, D, 0, torch.cuda.current_stream().cuda_stream)
    assert _lib.STATUS_NAMES[st] == "MGS_WORKSPACE_TOO_SMALL"
