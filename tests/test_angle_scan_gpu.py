"""GPU parity of the angle-fused Givens / rotation scan (fwd + bwd) against
the reference's golden vectors (GivensMinGRU / RotationMinGRU eager maths,
min_gru.py:2552-2602 and 2137-2155, scanned by matrix_affine_scan) and the
fp64 oracle (restatement of triton_scans.py:1038-1291).

Tolerances: fp32 forward rtol 1e-5 / atol 1e-6; gradients rtol 1e-4 /
atol 1e-5 (fp64 references); bf16 inputs with fp32 state rtol 2e-2."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import oracle

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


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


def _tol(base, ref):
    """atol relative to the magnitude the recurrence reaches: without decay the
    transitions are orthogonal (non-contractive), states grow like sqrt(t) and
    fp32 round-off -- in any fp32 implementation, the reference's included --
    grows with them, so the absolute floor scales with max|ref|."""
    return dict(rtol=base["rtol"], atol=base["atol"] * max(1.0, float(np.abs(ref).max())))


def check(got, ref_h, ref_g, has_scale, has_decay):
    h, dth, dsc, dga, db, dh0 = got
    np.testing.assert_allclose(h, ref_h, **_tol(FWD, ref_h))
    np.testing.assert_allclose(dth, ref_g["dtheta"], **_tol(BWD, ref_g["dtheta"]))
    np.testing.assert_allclose(db, ref_g["db"], **_tol(BWD, ref_g["db"]))
    np.testing.assert_allclose(dh0, ref_g["dh0"], **_tol(BWD, ref_g["dh0"]))
    if has_decay:
        np.testing.assert_allclose(dga, ref_g["dgamma"], **_tol(BWD, ref_g["dgamma"]))
    if has_scale:
        np.testing.assert_allclose(dsc, ref_g["dscale"], **_tol(BWD, ref_g["dscale"]))


@pytest.mark.parametrize("name", golden_names("givens_") + golden_names("rotation"))
def test_golden(cuda, name):
    g = load_golden(name)
    hs, hd = (int(x) for x in g["flags"])
    check(run(g, cuda, hs, hd), g["h"], g, hs, hd)


def make_inputs(B, T, n, R, k, seed, *, has_scale, has_decay, meta="brickwall"):
    import mingru_b200 as mb

    rng = np.random.default_rng(seed)
    d = {
        "theta": (rng.random((B, T, n, R, k // 2)) * 2 - 1) * math.pi,
        "scale": np.tanh(rng.standard_normal((B, T, n))) if has_scale else np.ones((B, T, n)),
        "gamma": 1 / (1 + np.exp(-rng.standard_normal((B, T, n)))) if has_decay else np.ones((B, T, n)),
        "b": rng.standard_normal((B, T, n, k)),
        "h0": rng.standard_normal((B, n, k)),
        "grad_h": rng.standard_normal((B, T, n, k)),
    }
    for key in ("theta", "scale", "gamma", "b", "h0", "grad_h"):
        d[key] = d[key].astype(np.float32).astype(np.float64)
    perm, sgn, p2p = (x.numpy() for x in mb.brickwall_meta(R, k))
    if meta == "shuffled":  # a valid pairing that is not the brick-wall layout
        perm, sgn, p2p = perm.copy(), sgn.copy(), p2p.copy()
        for r in range(R):
            order = rng.permutation(k)
            for m in range(k // 2):
                i, j = int(order[2 * m]), int(order[2 * m + 1])
                perm[r, i], perm[r, j] = j, i
                sgn[r, i], sgn[r, j] = -1.0, 1.0
                p2p[r, i], p2p[r, j] = m, m
    d.update(perm=perm, sgn=sgn, p2p=p2p)
    return d


def oracle_ref(d, has_scale, has_decay):
    kw = dict(has_scale=has_scale, has_decay=has_decay)
    h = oracle.angle_scan(d["theta"], d["scale"], d["gamma"], d["b"], d["h0"], d["perm"],
                          d["sgn"], d["p2p"], **kw)
    dth, dsc, dga, db, dh0 = oracle.angle_scan_bwd(
        d["theta"], d["scale"], d["gamma"], d["h0"], h, d["grad_h"], d["perm"], d["sgn"],
        d["p2p"], **kw)
    return h, {"dtheta": dth, "dscale": dsc, "dgamma": dga, "db": db, "dh0": dh0}


CASES = [  # (B, T, n, R, k, has_scale, has_decay, meta)
    (2, 13, 3, 1, 2, 1, 0, "brickwall"), (2, 100, 33, 1, 2, 1, 1, "brickwall"),
    (1, 64, 5, 2, 2, 0, 1, "brickwall"), (2, 37, 40, 3, 4, 0, 1, "brickwall"),
    (1, 50, 9, 4, 4, 0, 0, "brickwall"), (2, 70, 33, 2, 8, 0, 1, "brickwall"),
    (1, 45, 7, 3, 8, 0, 1, "brickwall"), (1, 23, 3, 4, 8, 0, 0, "brickwall"),
    (1, 20, 3, 3, 8, 0, 1, "shuffled"), (1, 15, 2, 2, 16, 0, 1, "brickwall"),
    (1, 9, 2, 5, 4, 0, 1, "brickwall"), (2, 1, 4, 2, 8, 0, 1, "brickwall"),
]


@pytest.mark.parametrize("case", CASES)
def test_vs_oracle(cuda, case):
    B, T, n, R, k, hs, hd, meta = case
    d = make_inputs(B, T, n, R, k, seed=sum(case[:5]), has_scale=hs, has_decay=hd, meta=meta)
    ref_h, ref_g = oracle_ref(d, hs, hd)
    check(run(d, cuda, hs, hd), ref_h, ref_g, hs, hd)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_inputs(cuda, dtype):
    d = make_inputs(2, 40, 9, 2, 8, seed=4, has_scale=0, has_decay=1)
    rnd = lambda x: torch.as_tensor(x, dtype=torch.float32).to(dtype).double().numpy()
    for key in ("theta", "scale", "gamma", "b", "h0", "grad_h"):
        d[key] = rnd(d[key])
    ref_h, ref_g = oracle_ref(d, 0, 1)
    h, dth, _, dga, db, dh0 = run(d, cuda, 0, 1, dtype)
    tol = dict(rtol=2e-2, atol=3e-2)
    np.testing.assert_allclose(h, ref_h, **tol)
    np.testing.assert_allclose(db, ref_g["db"], **tol)
    np.testing.assert_allclose(dh0, ref_g["dh0"], **tol)


def test_full_config4(cuda):
    """B=8, T=4096, n=128, k=8, R=2 with the wrap-around
    plane (7, 0) angle fixed to 0 (7 live nearest-neighbour rotations),
    gamma = sigmoid(N(0,1)), b ~ N(0,1), h0 = 0."""
    d = make_inputs(8, 4096, 128, 2, 8, seed=0, has_scale=0, has_decay=1)
    d["theta"][:, :, :, 1, 3] = 0.0
    d["h0"][:] = 0.0
    ref_h, ref_g = oracle_ref(d, 0, 1)
    check(run(d, cuda, 0, 1), ref_h, ref_g, 0, 1)
