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


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_inputs(cuda, dtype):
    d = make_inputs(2, 40, 9, 2, 8, seed=4, has_scale=0, has_decay=1)
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
