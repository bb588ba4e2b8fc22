"""GPU parity of the decay-active delta rule (DeltaMinGRU._forward_chunked_gated,
min_gru.py:3290-3448; the reference runs it in eager torch only) against the
reference's own outputs and gradients (tests/golden/deltagated_*.npz, made
through the reference's raw-tensor shim, with lambda and dt as inputs) and
against the sequential gated recurrence in float64 (oracle
delta_oracle.gated_sequential_torch, itself pinned to those fixtures by
tests/test_oracle.py).

Tolerances: the fp32 bar, forward rtol 1e-5 / atol 1e-6 and gradients
rtol 1e-4 / atol 1e-5, the absolute part raised to 10x the reference eager
path's own fp32-vs-fp64 deviation on the same inputs where that is larger
(the reference parity runner's rule, triton_scans.py:3303-3330; deviations in
tests/golden/eager_dev.json); lambda and dt gradients of the golden cases,
sums over the whole sequence, rtol 1e-4 / atol 1e-4; bf16 inputs rtol 2e-2 /
atol 2e-2 against the oracle on the bf16-rounded inputs."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import cases as C
from conftest import GOLDEN, golden_names, load_golden
from oracle import delta_oracle

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)
NAMES = ["dQ", "dK", "dV", "dbeta", "dH0"]
EAGER_DEV = json.loads((GOLDEN / "eager_dev.json").read_text())


def f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def run(d, lam, dtt, chunk, dev, dtype=torch.float32):
    import mingru_b200 as mb

    Q, K, V, beta = (torch.as_tensor(d[k], dtype=dtype, device=dev).requires_grad_(True)
                     for k in ("Q", "K", "V", "beta"))
    H0 = torch.as_tensor(d["H0"], dtype=torch.float32, device=dev).requires_grad_(True)
    tl = torch.as_tensor(lam, dtype=torch.float32, device=dev).requires_grad_(True)
    td = torch.as_tensor(dtt, dtype=torch.float32, device=dev).requires_grad_(True)
    lg = -tl[None, :, None] * td[:, None, :]
    y, HT = mb.delta_gated_scan_impl(Q, K, V, beta, H0, lg, chunk_size=chunk)
    torch.autograd.backward([y, HT], [torch.as_tensor(d["grad_y"], dtype=dtype, device=dev),
                                      torch.as_tensor(d["grad_H_T"], dtype=torch.float32, device=dev)])
    mb.raise_device_error(dev)
    return (f64(y), f64(HT), [f64(Q.grad), f64(K.grad), f64(V.grad), f64(beta.grad), f64(H0.grad)],
            f64(tl.grad), f64(td.grad))


@pytest.mark.parametrize("name", golden_names("deltagated_"))
def test_golden(cuda, name):
    g = load_golden(name)
    y, HT, grads, dlam, ddt = run(g, g["lam"], g["dt"], int(g["chunk"]), cuda)
    np.testing.assert_allclose(y, g["y"], **FWD)
    np.testing.assert_allclose(HT, g["H_T"], **FWD)
    for got, key in zip(grads, NAMES):
        np.testing.assert_allclose(got, g[key], **BWD, err_msg=key)
    np.testing.assert_allclose(dlam, g["dlam"], rtol=1e-4, atol=1e-4, err_msg="dlambda")
    np.testing.assert_allclose(ddt, g["ddt"], rtol=1e-4, atol=1e-4, err_msg="ddt")


def oracle_ref(d, lam, dtt):
    lg = -lam[None, :, None] * dtt[:, None, :]
    y, HT, grads = delta_oracle.gated_sequential_torch(d["Q"], d["K"], d["V"], d["beta"], d["H0"],
                                                       lg, d["grad_y"], d["grad_H_T"])
    dlg = grads[5]
    return y, HT, grads[:5], -(dlg * dtt[:, None, :]).sum((0, 2)), -(dlg * lam[None, :, None]).sum(1)


@pytest.mark.parametrize("case", C.DELTA_GATED_CASES)
def test_vs_oracle(cuda, case):
    d, lam, dtt = C.delta_gated_inputs(case, seed=sum(case))
    dev = EAGER_DEV[C.case_key("delta_gated", case)]
    ry, rHT, rg, rdlam, rddt = oracle_ref(d, lam, dtt)
    y, HT, grads, dlam, ddt = run(d, lam, dtt, case[-1], cuda)
    pairs = [("y", y, ry, FWD), ("H_T", HT, rHT, FWD)]
    pairs += [(k, g_, r_, BWD) for k, g_, r_ in zip(NAMES, grads, rg)]
    pairs += [("dlam", dlam, rdlam, BWD), ("ddt", ddt, rddt, BWD)]
    for name, g_, r_, _ in pairs:
        print(C.report(str(case), g_, r_, dev, name))
    for name, g_, r_, bar in pairs:
        np.testing.assert_allclose(g_, r_, **C.gate(bar, dev, name), err_msg=name)


def test_bf16_inputs(cuda):
    d, lam, dtt = C.delta_gated_inputs((1, 2, 80, 1, 32, 32, 32), seed=3)
    rnd = lambda x: torch.as_tensor(x, dtype=torch.float32).to(torch.bfloat16).double().numpy()
    for k in ("Q", "K", "V", "beta", "grad_y"):
        d[k] = rnd(d[k])
    ry, rHT, rg, rdlam, rddt = oracle_ref(d, lam, dtt)
    y, HT, grads, dlam, ddt = run(d, lam, dtt, 32, cuda, torch.bfloat16)
    tol = dict(rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(y, ry, **tol)
    np.testing.assert_allclose(HT, rHT, **tol)
    for got, ref, key in zip(grads, rg, NAMES):
        np.testing.assert_allclose(got, ref, **tol, err_msg=key)
    np.testing.assert_allclose(dlam, rdlam, **tol)
    np.testing.assert_allclose(ddt, rddt, **tol)


def test_zero_decay_equals_plain(cuda):
    """log gamma = 0 is the decay-free delta rule."""
    import mingru_b200 as mb

    d, lam, dtt = C.delta_gated_inputs((1, 2, 70, 1, 32, 32, 32), seed=8)
    t = lambda k: torch.as_tensor(d[k], dtype=torch.float32, device=cuda)
    args = (t("Q"), t("K"), t("V"), t("beta"), t("H0"))
    y0, H0 = mb.delta_scan_impl(*args, chunk_size=32)
    y1, H1 = mb.delta_gated_scan_impl(*args, torch.zeros(1, 2, 70, device=cuda), chunk_size=32)
    torch.testing.assert_close(y1, y0, **FWD)
    torch.testing.assert_close(H1, H0, **FWD)
