"""Sequence-parallel kernels on one GPU: the sequence is split into slices
and the per-slice operations (``mgs_*_carry_fwd/bwd`` summaries, prefix /
suffix composition, scans started from the carried-in state with
``mgs_*_fwd_fixup/bwd_fixup``) are run slice by slice, as each rank of a
sequence-parallel group would, with the all-gather replaced by stacking the
summaries. Every slice's outputs and input gradients must equal the
full-length scan's (one launch over the whole sequence) -- on the strip,
look-back (direct) and column paths of both scans.

Tolerances: fp32 forward rtol 1e-5 / atol 1e-6 (the slices reassociate the
scan, as the kernels' own tiles do), gradients rtol 1e-4 / atol 1e-5."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)

# (B, T, D, slices): strip path (B ceil(D/32) >= 2 x SMs), look-back path
# (narrow), ragged D on the look-back path
LINEAR = [(16, 4096, 1024, 4), (2, 1000, 36, 5), (3, 640, 37, 4), (20, 600, 1000, 3)]
# column path (T per slice <= 1024, many channel groups), strip path
# (T per slice > 1024), look-back path (narrow)
LOG = [(8, 4096, 256, 4), (20, 3000, 1024, 2), (2, 600, 40, 3), (16, 900, 120, 3)]


def _slices(T, n):
    per = T // n
    return [slice(r * per, (r + 1) * per) for r in range(n)]


@pytest.mark.parametrize("shape", LINEAR)
def test_linear_slices_equal_full_scan(cuda, shape):
    import mingru_b200 as mb
    from mingru_b200.parallel import KernelOps, linear_prefix, linear_suffix

    B, T, D, n = shape
    g = torch.Generator(device=cuda).manual_seed(sum(shape))
    a = torch.tanh(torch.randn(B, T, D, device=cuda, generator=g))
    b = torch.randn(B, T, D, device=cuda, generator=g)
    gA = torch.randn(B, T, D, device=cuda, generator=g)
    gB = torch.randn(B, T, D, device=cuda, generator=g)
    ta, tb = a.clone().requires_grad_(True), b.clone().requires_grad_(True)
    A, Bc = mb.linear_scan(ta, tb)
    torch.autograd.backward([A, Bc], [gA, gB])

    ops = KernelOps()
    sl = _slices(T, n)
    G = torch.stack([ops.linear_carry_fwd(a[:, s], b[:, s]) for s in sl])
    R = torch.stack([ops.linear_carry_bwd(a[:, s], gA[:, s], gB[:, s]) for s in sl])
    for r, s in enumerate(sl):
        As, Bs, car = ops.linear_fwd_fixup(a[:, s], b[:, s], linear_prefix(G, r))
        torch.testing.assert_close(As, A[:, s], **FWD)
        torch.testing.assert_close(Bs, Bc[:, s], **FWD)
        da, db = ops.linear_bwd_fixup(a[:, s], b[:, s], car, linear_suffix(R, r), gA[:, s], gB[:, s])
        torch.testing.assert_close(da, ta.grad[:, s], **BWD)
        torch.testing.assert_close(db, tb.grad[:, s], **BWD)
    mb.raise_device_error(cuda)


@pytest.mark.parametrize("shape", LOG)
def test_log_slices_equal_full_scan(cuda, shape):
    import mingru_b200 as mb
    from mingru_b200.parallel import KernelOps, log_prefix, log_suffix

    B, T, D, n = shape
    g = torch.Generator(device=cuda).manual_seed(sum(shape))
    k = torch.randn(B, T, D, device=cuda, generator=g)
    x = torch.randn(B, T, D, device=cuda, generator=g)
    lc = -torch.nn.functional.softplus(k)
    lv = torch.cat([torch.full((B, 1, D), -0.7, device=cuda),
                    -torch.nn.functional.softplus(-k) + mb.log_g(x)], 1)
    gh = torch.randn(B, T, D, device=cuda, generator=g)
    tlc, tlv = lc.clone().requires_grad_(True), lv.clone().requires_grad_(True)
    h = mb.parallel_scan_log(tlc, tlv)
    h.backward(gh)

    ops = KernelOps()
    sl = _slices(T, n)
    lvs = [lv[:, s.start:s.stop + 1] for s in sl]  # slot 0 = previous row (unused for r > 0)
    G = torch.stack([torch.cat([ops.log_carry_fwd(lc[:, s], lvs[r]), lvs[r][:, 0].float()[None]])
                     for r, s in enumerate(sl)])
    R = torch.stack([ops.log_carry_bwd(lc[:, s], gh[:, s]) for s in sl])
    for r, s in enumerate(sl):
        lh_in = log_prefix(G, r)
        hs, car = ops.log_fwd_fixup(lc[:, s], lvs[r], lh_in)
        torch.testing.assert_close(hs, h[:, s], **FWD)
        dlc, dlv = ops.log_bwd_fixup(lc[:, s], lvs[r], lh_in, car, log_suffix(R, r), gh[:, s])
        torch.testing.assert_close(dlc, tlc.grad[:, s], **BWD)
        torch.testing.assert_close(dlv[:, 1:], tlv.grad[:, s.start + 1:s.stop + 1], **BWD)
        if r == 0:
            torch.testing.assert_close(dlv[:, 0], tlv.grad[:, 0], **BWD)
    mb.raise_device_error(cuda)
