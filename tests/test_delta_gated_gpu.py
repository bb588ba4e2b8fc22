"""GPU parity of the decay-active delta rule (DeltaMinGRU._forward_chunked_gated,
min_gru.py:3290-3448; the reference runs it in eager torch only) against the
reference's own outputs and gradients (tests/golden/deltagated_*.npz, made
through the reference's raw-tensor shim, with lambda and dt as inputs) and
against the sequential gated recurrence in float64 (oracle
delta_oracle.gated_sequential_torch, itself pinned to those fixtures by
tests/test_oracle.py).

Tolerances: the fp32 bar, forward rtol 1e-5 / atol 1e-6 and gradients
rtol 1e-4 / atol 1e-5 (lambda and dt gradients sum over the sequence: atol
1e-4); bf16 inputs rtol 2e-2 / atol 2e-2 against the oracle on the
bf16-rounded inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import delta_oracle

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)
NAMES = ["dQ", "dK", "dV", "dbeta", "dH0"]


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


def make(B, H, T, nh, dk, dv, seed):
    rng = np.random.default_rng(seed)
    K = rng.standard_normal((B, H, T, nh, dk))
    K /= np.linalg.norm(K, axis=-1, keepdims=True)
    d = {
        "Q": rng.standard_normal((B, H, T, dk)),
        "K": K,
        "V": rng.standard_normal((B, H, T, nh, dv)),
        "beta": 2 / (1 + np.exp(-rng.standard_normal((B, H, T, nh)))),
        "H0": rng.standard_normal((B, H, dk, dv)) * 0.1,
        "grad_y": rng.standard_normal((B, H, T, dv)),
        "grad_H_T": rng.standard_normal((B, H, dk, dv)),
    }
    lam = rng.random(H) * 0.5 + 0.05
    dtt = rng.random((B, T)) * 2
    dtt[:, T // 3] = 1e3  # one saturated gap: memory wiped there
    f32 = lambda a: np.asarray(a).astype(np.float32).astype(np.float64)
    return {k: f32(v) for k, v in d.items()}, f32(lam), f32(dtt)


def oracle_ref(d, lam, dtt):
    lg = -lam[None, :, None] * dtt[:, None, :]
    y, HT, grads = delta_oracle.gated_sequential_torch(d["Q"], d["K"], d["V"], d["beta"], d["H0"],
                                                       lg, d["grad_y"], d["grad_H_T"])
    dlg = grads[5]
    return y, HT, grads[:5], -(dlg * dtt[:, None, :]).sum((0, 2)), -(dlg * lam[None, :, None]).sum(1)


CASES = [  # (B, H, T, nh, dk, dv, chunk)
    (2, 2, 100, 1, 32, 32, 32), (1, 2, 150, 2, 16, 16, 64), (1, 1, 70, 1, 64, 64, 64),
    (2, 3, 45, 3, 8, 16, 10), (1, 2, 90, 1, 16, 80, 64),
]


@pytest.mark.parametrize("case", CASES)
def test_vs_oracle(cuda, case):
    d, lam, dtt = make(*case[:6], seed=sum(case))
    ry, rHT, rg, rdlam, rddt = oracle_ref(d, lam, dtt)
    y, HT, grads, dlam, ddt = run(d, lam, dtt, case[-1], cuda)
    np.testing.assert_allclose(y, ry, **FWD)
    np.testing.assert_allclose(HT, rHT, **FWD)
    for got, ref, key in zip(grads, rg, NAMES):
        np.testing.assert_allclose(got, ref, **BWD, err_msg=key)
    np.testing.assert_allclose(dlam, rdlam, rtol=1e-4, atol=1e-4, err_msg="dlambda")
    np.testing.assert_allclose(ddt, rddt, rtol=1e-4, atol=1e-4, err_msg="ddt")


def test_bf16_inputs(cuda):
    d, lam, dtt = make(1, 2, 80, 1, 32, 32, seed=3)
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

    d, lam, dtt = make(1, 2, 70, 1, 32, 32, seed=8)
    t = lambda k: torch.as_tensor(d[k], dtype=torch.float32, device=cuda)
    args = (t("Q"), t("K"), t("V"), t("beta"), t("H0"))
    y0, H0 = mb.delta_scan_impl(*args, chunk_size=32)
    y1, H1 = mb.delta_gated_scan_impl(*args, torch.zeros(1, 2, 70, device=cuda), chunk_size=32)
    torch.testing.assert_close(y1, y0, **FWD)
    torch.testing.assert_close(H1, H0, **FWD)
