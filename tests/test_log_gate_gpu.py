"""GPU parity of the MinGRU gate scan (parallel_scan_log fed from the gate and
candidate pre-activations, the coefficient prologue of MinGRU.forward,
min_gru.py:1383-1397, fused into the scan kernels) against the fp64 oracle
(oracle.mingru_gate_scan: the prologue restated in numpy, then the
sequential log-space recurrence and its adjoint) and against the unfused
path (parallel_scan_log on coefficients built by torch).

Tolerances: fp32 forward rtol 1e-5 / atol 1e-6, gradients rtol 1e-4 /
atol 1e-5; bf16 storage rtol 2e-2 / atol 2e-2 against the oracle on the
bf16-rounded inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


def f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def inputs(B, T, D, seed, extreme=False):
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((B, T, D))
    x = rng.standard_normal((B, T, D))
    if extreme:  # saturated gates, x~ exactly 0, tiny and large candidates
        k.flat[::7] = 60.0
        k.flat[3::7] = -60.0
        x.flat[::5] = 0.0
        x.flat[1::11] = 1e-30
        x.flat[2::13] = -1e-30
        x.flat[4::17] = 40.0
    lh0 = np.log(np.full((B, D), 0.5)) + 0.1 * rng.standard_normal((B, D))
    gh = rng.standard_normal((B, T, D))
    f32 = lambda a: a.astype(np.float32).astype(np.float64)
    return f32(k), f32(x), f32(lh0), f32(gh)


def run(k, x, lh0, gh, dev, dtype=torch.float32):
    import mingru_b200 as mb

    tk, tx, tl = (torch.as_tensor(a, dtype=dtype, device=dev).requires_grad_(True)
                  for a in (k, x, lh0))
    h = mb.mingru_gate_scan(tk, tx, tl)
    h.backward(torch.as_tensor(gh, dtype=dtype, device=dev))
    mb.raise_device_error(dev)
    return f64(h), f64(tk.grad), f64(tx.grad), f64(tl.grad)


# column path (fused prologue): (8, 1024, 256) is BASELINE config 1's shape,
# (10, 1024, 124) ends in a partial 8-channel group, (160, 1, 64) has T = 1;
# elementwise-prologue routes: (2, 300, 256) direct look-back tiles,
# (3, 2000, 256) T above the column bound, (20, 1500, 1024) the strip path.
SHAPES = [(8, 1024, 256), (16, 200, 128), (10, 1024, 124), (160, 1, 64), (2, 300, 256),
          (3, 2000, 256), (20, 1500, 1024), (1, 37, 5)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("extreme", [False, True])
def test_vs_oracle(cuda, shape, extreme):
    k, x, lh0, gh = inputs(*shape, seed=sum(shape), extreme=extreme)
    h, dk, dx, dl = run(k, x, lh0, gh, cuda)
    rh = oracle.mingru_gate_scan(k, x, lh0)
    rdk, rdx, rdl = oracle.mingru_gate_scan_bwd(k, x, lh0, gh)
    np.testing.assert_allclose(h, rh, **FWD)
    np.testing.assert_allclose(dk, rdk, **BWD, err_msg="dk")
    np.testing.assert_allclose(dx, rdx, **BWD, err_msg="dx")
    np.testing.assert_allclose(dl, rdl, **BWD, err_msg="dlog_h0")


def test_matches_unfused(cuda):
    """Same numbers as parallel_scan_log on the coefficients torch builds."""
    import mingru_b200 as mb

    k, x, lh0, gh = inputs(8, 1024, 256, seed=3)
    tk, tx, tl = (torch.as_tensor(a, dtype=torch.float32, device=cuda).requires_grad_(True)
                  for a in (k, x, lh0))
    lc = -F.softplus(tk)
    lv = torch.cat([tl[:, None], -F.softplus(-tk) + mb.log_g(tx)], 1)
    h_ref = mb.parallel_scan_log(lc, lv)
    g_ref = torch.autograd.grad(h_ref, (tk, tx, tl), torch.as_tensor(gh, dtype=torch.float32,
                                                                      device=cuda))
    h = mb.mingru_gate_scan(tk, tx, tl)
    g = torch.autograd.grad(h, (tk, tx, tl), torch.as_tensor(gh, dtype=torch.float32, device=cuda))
    torch.testing.assert_close(h, h_ref, **FWD)
    for a, b in zip(g, g_ref):
        torch.testing.assert_close(a, b, **BWD)


@pytest.mark.parametrize("shape", [(8, 512, 256), (2, 300, 40)])
def test_bf16_storage(cuda, shape):
    k, x, lh0, gh = inputs(*shape, seed=11)
    rnd = lambda a: torch.as_tensor(a, dtype=torch.float32).to(torch.bfloat16).double().numpy()
    k, x, lh0, gh = rnd(k), rnd(x), rnd(lh0), rnd(gh)
    h, dk, dx, dl = run(k, x, lh0, gh, cuda, torch.bfloat16)
    rh = oracle.mingru_gate_scan(k, x, lh0)
    rdk, rdx, rdl = oracle.mingru_gate_scan_bwd(k, x, lh0, gh)
    tol = dict(rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(h, rh, **tol)
    np.testing.assert_allclose(dk, rdk, **tol)
    np.testing.assert_allclose(dx, rdx, **tol)
    np.testing.assert_allclose(dl, rdl, **tol)


def test_empty_time_axis(cuda):
    import mingru_b200 as mb

    k = torch.zeros(2, 0, 8, device=cuda, requires_grad=True)
    lh0 = torch.zeros(2, 8, device=cuda, requires_grad=True)
    h = mb.mingru_gate_scan(k, k, lh0)
    assert h.shape == (2, 0, 8)
    (g,) = torch.autograd.grad(h.sum(), (lh0,), allow_unused=True, materialize_grads=True)
    assert torch.count_nonzero(g) == 0
