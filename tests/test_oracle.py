"""Pin the CPU oracle to the reference: every golden vector produced by the
reference's own eager code (tests/golden/make_golden.py) must be reproduced by
the oracle's sequential restatements to fp64 round-off."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_names, load_golden
from oracle import delta_oracle, oracle

RT, AT = 1e-9, 1e-11


def close(x, y):
    np.testing.assert_allclose(x, y, rtol=RT, atol=AT)


@pytest.mark.parametrize("name", golden_names("log_"))
def test_log_scan_matches_reference(name):
    g = load_golden(name)
    close(oracle.parallel_scan_log(g["log_coeffs"], g["log_values"]), g["h"])
    dlc, dlv = oracle.parallel_scan_log_bwd(g["log_coeffs"], g["log_values"], g["grad_h"])
    close(dlc, g["dlog_coeffs"])
    close(dlv, g["dlog_values"])


@pytest.mark.parametrize("name", golden_names("linear_"))
def test_linear_scan_matches_reference(name):
    g = load_golden(name)
    A, Bc = oracle.linear_scan(g["a"], g["b"])
    close(A, g["A"])
    close(Bc, g["Bc"])
    da, db = oracle.linear_scan_bwd(g["a"], A, Bc, g["gA"], g["gBc"])
    close(da, g["da"])
    close(db, g["db"])


@pytest.mark.parametrize("name", golden_names("matrix_"))
def test_matrix_scan_matches_reference(name):
    g = load_golden(name)
    A, Bc = oracle.matrix_scan(g["M"], g["b"])
    close(A, g["A"])
    close(Bc, g["Bc"])
    dM, db = oracle.matrix_scan_bwd(g["M"], A, Bc, g["gA"], g["gBc"])
    close(dM, g["dM"])
    close(db, g["db"])


@pytest.mark.parametrize("name", golden_names("affine_"))
def test_affine_scan_matches_reference(name):
    g = load_golden(name)
    Ab, Bb = oracle.matrix_affine_scan(g["A"], g["Bm"])
    close(Ab, g["Abar"])
    close(Bb, g["Bbar"])
    dA, dB = oracle.matrix_affine_scan_bwd(g["A"], Ab, Bb, g["gAbar"], g["gBbar"])
    close(dA, g["dA"])
    close(dB, g["dBm"])


@pytest.mark.parametrize("name", golden_names("givens_") + golden_names("rotation"))
def test_angle_scan_matches_reference(name):
    g = load_golden(name)
    has_scale, has_decay = (int(x) for x in g["flags"])
    kw = dict(has_scale=has_scale, has_decay=has_decay)
    h = oracle.angle_scan(g["theta"], g["scale"], g["gamma"], g["b"], g["h0"], g["perm"],
                          g["sgn"], g["p2p"], **kw)
    close(h, g["h"])
    dth, dsc, dga, db, dh0 = oracle.angle_scan_bwd(
        g["theta"], g["scale"], g["gamma"], g["h0"], h, g["grad_h"], g["perm"], g["sgn"],
        g["p2p"], **kw)
    close(dth, g["dtheta"])
    close(db, g["db"])
    close(dh0, g["dh0"])
    if has_decay:
        close(dga, g["dgamma"])
    if has_scale:
        close(dsc, g["dscale"])


@pytest.mark.parametrize("name", golden_names("delta_"))
def test_delta_matches_reference(name):
    g = load_golden(name)
    c = int(g["chunk"])
    y, HT = delta_oracle.delta_forward(g["Q"], g["K"], g["V"], g["beta"], g["H0"], c)
    close(y, g["y"])
    close(HT, g["H_T"])
    ys, HTs = delta_oracle.delta_sequential(g["Q"], g["K"], g["V"], g["beta"], g["H0"])
    np.testing.assert_allclose(ys, g["y"], rtol=1e-8, atol=1e-9)
    np.testing.assert_allclose(HTs, g["H_T"], rtol=1e-8, atol=1e-9)
    grads = delta_oracle.delta_backward(g["Q"], g["K"], g["V"], g["beta"], g["H0"],
                                        g["grad_y"], g["grad_H_T"], c)
    for got, key in zip(grads, ["dQ", "dK", "dV", "dbeta", "dH0"]):
        np.testing.assert_allclose(got, g[key], rtol=1e-8, atol=1e-9)


def test_float32_oracle_tracks_float64():
    rng = np.random.default_rng(0)
    a = np.tanh(rng.standard_normal((2, 300, 8)))
    b = rng.standard_normal((2, 300, 8))
    A64, B64 = oracle.linear_scan(a, b)
    A32, B32 = oracle.linear_scan(a, b, dtype=np.float32)
    np.testing.assert_allclose(B32, B64, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(A32, A64, rtol=1e-4, atol=1e-30)


@pytest.mark.parametrize("name", golden_names("deltagated_"))
def test_gated_delta_oracle_vs_reference(name):
    """The sequential gated recurrence (oracle.delta_oracle.gated_sequential_torch)
    reproduces the reference's chunked _forward_chunked_gated and its autograd
    gradients, including those w.r.t. lambda and dt (log gamma = -lambda dt)."""
    from oracle import delta_oracle

    g = load_golden(name)
    lam, dtt = g["lam"], g["dt"]
    lg = -lam[None, :, None] * dtt[:, None, :]
    y, HT, grads = delta_oracle.gated_sequential_torch(
        g["Q"], g["K"], g["V"], g["beta"], g["H0"], lg, g["grad_y"], g["grad_H_T"])
    tol = dict(rtol=1e-9, atol=1e-10)
    np.testing.assert_allclose(y, g["y"], **tol)
    np.testing.assert_allclose(HT, g["H_T"], **tol)
    for got, key in zip(grads[:5], ["dQ", "dK", "dV", "dbeta", "dH0"]):
        np.testing.assert_allclose(got, g[key], **tol, err_msg=key)
    dlg = grads[5]
    np.testing.assert_allclose(-(dlg * dtt[:, None, :]).sum((0, 2)), g["dlam"], **tol)
    np.testing.assert_allclose(-(dlg * lam[None, :, None]).sum(1), g["ddt"], **tol)
