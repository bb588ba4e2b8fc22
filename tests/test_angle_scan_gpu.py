"""GPU parity of the angle-fused Givens / rotation scan (fwd + bwd) against
the reference's golden vectors (GivensMinGRU / RotationMinGRU eager maths,
min_gru.py:2552-2602 and 2137-2155, scanned by matrix_affine_scan) and the
fp64 oracle (restatement of triton_scans.py:1038-1291).

Tolerances: the parity bar, fp32 forward rtol 1e-5 / atol 1e-6 and gradients
rtol 1e-4 / atol 1e-5 (fp64 references); bf16 inputs with fp32 state
rtol 2e-2. Where the reference's own eager path deviates more between fp32
and fp64 on the same inputs (without decay the transitions are orthogonal,
the states grow and fp32 round-off grows with them, in any implementation),
the absolute part is 10x that deviation -- the reference parity runner's
rule (triton_scans.py:3303-3330), deviations from tests/golden/eager_dev.json
(tests/golden/make_golden.py --eager-dev, inputs from tests/cases.py). Every
comparison prints |kernel - fp64|, |eager32 - fp64| and their ratio."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import cases as C
from conftest import GOLDEN, golden_names, load_golden
from oracle import oracle

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)

EAGER_DEV = json.loads((GOLDEN / "eager_dev.json").read_text())


def f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def run(inp, dev, has_scale, has_decay, dtype=torch.float32):
    import mingru_b200 as mb

    th, sc, ga, bb, h0 = (torch.as_tensor(inp[k], dtype=dtype, device=dev).requires_grad_(True)
                          for k in ("theta", "scale", "gamma", "b", "h0"))
    perm = torch.as_tensor(inp["perm"], dtype=torch.int32, device=dev)
    sgn = torch.as_tensor(inp["sgn"], dtype=torch.float32, device=dev)
    p2p = torch.as_tensor(inp["p2p"], dtype=torch.int32, device=dev)
    h = mb.angle_scan_impl(th, sc, ga, bb, h0, perm, sgn, p2p,
                           has_scale=has_scale, has_decay=has_decay)
    h.backward(torch.as_tensor(inp["grad_h"], dtype=dtype, device=dev))
    mb.raise_device_error(dev)
    return f64(h), f64(th.grad), f64(sc.grad), f64(ga.grad), f64(bb.grad), f64(h0.grad)


def check(got, ref_h, ref_g, has_scale, has_decay, dev=None, label=""):
    h, dth, dsc, dga, db, dh0 = got
    pairs = [("h", h, ref_h, FWD), ("dtheta", dth, ref_g["dtheta"], BWD),
             ("db", db, ref_g["db"], BWD), ("dh0", dh0, ref_g["dh0"], BWD)]
    if has_decay:
        pairs.append(("dgamma", dga, ref_g["dgamma"], BWD))
    if has_scale:
        pairs.append(("dscale", dsc, ref_g["dscale"], BWD))
    for name, g, r, _ in pairs:
        print(C.report(label, g, r, dev, name))
    for name, g, r, bar in pairs:
        np.testing.assert_allclose(g, r, **C.gate(bar, dev, name), err_msg=f"{label} {name}")


@pytest.mark.parametrize("name", golden_names("givens_") + golden_names("rotation"))
def test_golden(cuda, name):
    g = load_golden(name)
    hs, hd = (int(x) for x in g["flags"])
    check(run(g, cuda, hs, hd), g["h"], g, hs, hd, EAGER_DEV["golden:" + name], name)


def make_inputs(B, T, n, R, k, seed, *, has_scale, has_decay, meta="brickwall"):
    return C.angle_inputs(B, T, n, R, k, seed, has_scale=has_scale, has_decay=has_decay, meta=meta)


def oracle_ref(d, has_scale, has_decay):
    kw = dict(has_scale=has_scale, has_decay=has_decay)
    h = oracle.angle_scan(d["theta"], d["scale"], d["gamma"], d["b"], d["h0"], d["perm"],
                          d["sgn"], d["p2p"], **kw)
    dth, dsc, dga, db, dh0 = oracle.angle_scan_bwd(
        d["theta"], d["scale"], d["gamma"], d["h0"], h, d["grad_h"], d["perm"], d["sgn"],
        d["p2p"], **kw)
    return h, {"dtheta": dth, "dscale": dsc, "dgamma": dga, "db": db, "dh0": dh0}


@pytest.mark.parametrize("case", C.ANGLE_CASES)
def test_vs_oracle(cuda, case):
    hs, hd = case[5], case[6]
    d = C.angle_case_inputs(case)
    ref_h, ref_g = oracle_ref(d, hs, hd)
    check(run(d, cuda, hs, hd), ref_h, ref_g, hs, hd, EAGER_DEV[C.case_key("angle", case)],
          str(case))


# Wider lane groups of the fast kernels: a partial last group of 128 lanes
# spanning two batch rows, k = 4, R = 3 with a ragged last tile, and a scale.
# The states stay bounded (decay), so fp32 meets the bar directly.
WIDE_CASES = [(3, 300, 68, 2, 8, 0, 1), (2, 200, 64, 2, 4, 0, 1), (1, 257, 128, 3, 8, 0, 1),
              (2, 150, 72, 2, 8, 1, 1)]


@pytest.mark.parametrize("case", WIDE_CASES)
def test_wide_groups_vs_oracle(cuda, case):
    B, T, n, R, k, hs, hd = case
    d = make_inputs(B, T, n, R, k, seed=sum(case), has_scale=hs, has_decay=hd)
    ref_h, ref_g = oracle_ref(d, hs, hd)
    check(run(d, cuda, hs, hd), ref_h, ref_g, hs, hd, None, str(case))


@pytest.mark.parametrize("n", [9, 72])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_inputs(cuda, dtype, n):
    d = make_inputs(2, 40, n, 2, 8, seed=4, has_scale=0, has_decay=1)
    rnd = lambda x: torch.as_tensor(x, dtype=torch.float32).to(dtype).double().numpy()
    for key in ("theta", "scale", "gamma", "b", "h0", "grad_h"):
        d[key] = rnd(d[key])
    ref_h, ref_g = oracle_ref(d, 0, 1)
    h, dth, _, dga, db, dh0 = run(d, cuda, 0, 1, dtype)
    tol = dict(rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(h, ref_h, **tol)
    np.testing.assert_allclose(db, ref_g["db"], **tol)
    np.testing.assert_allclose(dh0, ref_g["dh0"], **tol)


def test_full_config4(cuda):
    """B=8, T=4096, n=128, k=8, R=2 with the wrap-around
    plane (7, 0) angle fixed to 0 (7 live nearest-neighbour rotations),
    gamma = sigmoid(N(0,1)), b ~ N(0,1), h0 = 0. The eager deviation was
    measured on the first batch row (the rows are i.i.d.)."""
    d = C.angle_full_config4()
    ref_h, ref_g = oracle_ref(d, 0, 1)
    check(run(d, cuda, 0, 1), ref_h, ref_g, 0, 1, EAGER_DEV["angle_full_config4"], "config4")


@pytest.mark.parametrize("hs,hd", [(0, 1), (1, 1), (0, 0)])
def test_forward_without_grad(cuda, hs, hd):
    """A forward with nothing to differentiate keeps the tiles' linear parts
    in the workspace instead of the saved carries; its output must be the
    same bits as the autograd forward's (and meet the oracle)."""
    import mingru_b200 as mb

    k, R = (2, 1) if hs else (8, 2)
    d = make_inputs(3, 700, 45, R, k, seed=11, has_scale=hs, has_decay=hd)
    t = lambda key: torch.as_tensor(d[key], dtype=torch.float32, device=cuda)
    args = [t(x) for x in ("theta", "scale", "gamma", "b", "h0")]
    meta = [torch.as_tensor(d["perm"], dtype=torch.int32, device=cuda),
            torch.as_tensor(d["sgn"], dtype=torch.float32, device=cuda),
            torch.as_tensor(d["p2p"], dtype=torch.int32, device=cuda)]
    with torch.no_grad():
        h_ng = mb.angle_scan_impl(*args, *meta, has_scale=hs, has_decay=hd)
    h_g = mb.angle_scan_impl(*[a.clone().requires_grad_(True) for a in args], *meta,
                             has_scale=hs, has_decay=hd)
    mb.raise_device_error(cuda)
    assert torch.equal(h_ng, h_g.detach())
    if hd:  # with decay the states stay bounded and fp32 meets the forward bar
        ref_h, _ = oracle_ref(d, hs, hd)
        np.testing.assert_allclose(f64(h_ng), ref_h, **FWD)


def test_step_angles_match_fp64(cuda):
    """One step of a k=2, R=1 rotation from h0 = (1, 0) with b = 0 and no
    decay returns (cos theta, sin theta) exactly as the fast kernels compute
    them (their own reduction by pi/2 and polynomials; sincosf beyond
    |theta| > 8192). Bars: absolute error <= 2^-23 against fp64 on the
    polynomial range (the method's bound is 1.3 * 2^-24), <= 2^-22 where
    sincosf takes over, and within 2^-22 of CUDA's own fp32 sin / cos."""
    import math

    import mingru_b200 as mb

    g = torch.Generator().manual_seed(5)
    k = torch.arange(-5000, 5001, dtype=torch.float64)
    parts = [
        (torch.rand(1 << 18, generator=g, dtype=torch.float64) * 2 - 1) * math.pi,
        (torch.rand(1 << 16, generator=g, dtype=torch.float64) * 2 - 1) * 8192,
        k * math.pi / 2, (k + 0.5) * math.pi / 2,
        torch.tensor([0.0, -0.0, 1e-30, -1e-30, 8191.9, -8191.9]),
    ]
    fast = torch.cat(parts).float()
    wide = torch.cat([(torch.rand(4096, generator=g, dtype=torch.float64) * 2 - 1) * 1e6,
                      torch.tensor([8192.5, -8192.5, 1e20, -3e38])]).float()
    theta = torch.cat([fast, wide])
    n = theta.numel()
    th = theta.to(cuda).view(1, 1, n, 1, 1)
    ones = torch.ones(1, 1, n, device=cuda)
    b = torch.zeros(1, 1, n, 2, device=cuda)
    h0 = torch.zeros(1, n, 2, device=cuda)
    h0[..., 0] = 1.0
    perm, sgn, p2p = (torch.as_tensor(x, device=cuda) for x in C.brickwall(1, 2))
    h = mb.angle_scan_impl(th, ones, ones, b, h0, perm.int(), sgn.float(), p2p.int(),
                           has_scale=0, has_decay=0)
    mb.raise_device_error(cuda)
    got_c, got_s = h[0, 0, :, 0].double().cpu(), h[0, 0, :, 1].double().cpu()
    t64 = theta.double()
    ec, es = (got_c - torch.cos(t64)).abs(), (got_s - torch.sin(t64)).abs()
    nf = fast.numel()
    print(f"fast range: max |cos err| {ec[:nf].max():.3e}, |sin err| {es[:nf].max():.3e}; "
          f"sincosf range: {ec[nf:].max():.3e}, {es[nf:].max():.3e}")
    assert ec[:nf].max() <= 2.0 ** -23 and es[:nf].max() <= 2.0 ** -23
    assert ec[nf:].max() <= 2.0 ** -22 and es[nf:].max() <= 2.0 ** -22
    tc = th.view(-1)
    dc = (h[0, 0, :, 0] - torch.cos(tc)).abs().max().item()
    ds = (h[0, 0, :, 1] - torch.sin(tc)).abs().max().item()
    print(f"against CUDA fp32 cos / sin: {dc:.3e} {ds:.3e}")
    assert dc <= 2.0 ** -22 and ds <= 2.0 ** -22
