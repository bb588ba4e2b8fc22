"""GPU parity of the DeltaMinGRU chunked-WY delta rule (fwd + bwd) against the
reference's golden vectors (DeltaMinGRU._forward_chunked through the
reference's raw-tensor shim, min_gru.py:3152-3255) and the fp64 oracle
(chunked restatement + the sequential micro-step recurrence).

Tolerances: fp32 forward rtol 1e-5 / atol 1e-5 and gradients rtol 1e-4 /
atol 1e-4 against fp64 (the unit-triangular solves and the chunk-state chain
accumulate O(T/chunk) rounding steps); bf16 inputs with fp32 state rtol 2e-2."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import delta_oracle

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-5)
BWD = dict(rtol=1e-4, atol=1e-4)


def f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def run(d, chunk, dev, dtype=torch.float32):
    import mingru_b200 as mb

    Q, K, V, beta = (torch.as_tensor(d[k], dtype=dtype, device=dev).requires_grad_(True)
                     for k in ("Q", "K", "V", "beta"))
    H0 = torch.as_tensor(d["H0"], dtype=torch.float32, device=dev).requires_grad_(True)
    y, HT = mb.delta_scan_impl(Q, K, V, beta, H0, chunk_size=chunk)
    torch.autograd.backward([y, HT], [torch.as_tensor(d["grad_y"], dtype=dtype, device=dev),
                                      torch.as_tensor(d["grad_H_T"], dtype=torch.float32, device=dev)])
    return f64(y), f64(HT), f64(Q.grad), f64(K.grad), f64(V.grad), f64(beta.grad), f64(H0.grad)


NAMES = ["dQ", "dK", "dV", "dbeta", "dH0"]


@pytest.mark.parametrize("name", golden_names("delta_"))
def test_golden(cuda, name):
    g = load_golden(name)
    y, HT, *grads = run(g, int(g["chunk"]), cuda)
    np.testing.assert_allclose(y, g["y"], **FWD)
    np.testing.assert_allclose(HT, g["H_T"], **FWD)
    for got, key in zip(grads, NAMES):
        np.testing.assert_allclose(got, g[key], **BWD, err_msg=key)


def make(B, H, T, nh, dk, dv, seed):
    rng = np.random.default_rng(seed)
    K = rng.standard_normal((B, H, T, nh, dk))
    K /= np.linalg.norm(K, axis=-1, keepdims=True)
    d = {
        "Q": rng.standard_normal((B, H, T, dk)),
        "K": K,
        "V": rng.standard_normal((B, H, T, nh, dv)),
        "beta": 1 / (1 + np.exp(-rng.standard_normal((B, H, T, nh)))),
        "H0": rng.standard_normal((B, H, dk, dv)) * 0.1,
        "grad_y": rng.standard_normal((B, H, T, dv)),
        "grad_H_T": rng.standard_normal((B, H, dk, dv)),
    }
    return {k: v.astype(np.float32).astype(np.float64) for k, v in d.items()}


def oracle_ref(d, chunk):
    y, HT = delta_oracle.delta_forward(d["Q"], d["K"], d["V"], d["beta"], d["H0"], chunk)
    grads = delta_oracle.delta_backward(d["Q"], d["K"], d["V"], d["beta"], d["H0"],
                                        d["grad_y"], d["grad_H_T"], chunk)
    return y, HT, grads


CASES = [  # (B, H, T, nh, dk, dv, chunk)
    (1, 2, 100, 1, 64, 64, 64), (2, 1, 77, 2, 32, 32, 32), (1, 2, 130, 1, 16, 16, 16),
    (2, 2, 19, 1, 8, 8, 8), (1, 1, 65, 1, 64, 32, 64), (1, 3, 40, 4, 8, 16, 16),
    (1, 1, 1, 1, 4, 4, 4),
]


@pytest.mark.parametrize("case", CASES)
def test_vs_oracle(cuda, case):
    B, H, T, nh, dk, dv, chunk = case
    d = make(B, H, T, nh, dk, dv, seed=sum(case))
    ry, rHT, rg = oracle_ref(d, chunk)
    y, HT, *grads = run(d, chunk, cuda)
    np.testing.assert_allclose(y, ry, **FWD)
    np.testing.assert_allclose(HT, rHT, **FWD)
    for got, ref, key in zip(grads, rg, NAMES):
        np.testing.assert_allclose(got, ref, **BWD, err_msg=key)


def test_bf16_inputs_fp32_state(cuda):
    d = make(1, 2, 200, 1, 64, 64, seed=9)
    rnd = lambda x: torch.as_tensor(x, dtype=torch.float32).to(torch.bfloat16).double().numpy()
    for k in ("Q", "K", "V", "beta", "grad_y"):
        d[k] = rnd(d[k])
    ry, rHT, rg = oracle_ref(d, 64)
    y, HT, *grads = run(d, 64, cuda, torch.bfloat16)
    tol = dict(rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(y, ry, **tol)
    np.testing.assert_allclose(HT, rHT, **tol)
    for got, ref, key in zip(grads, rg, NAMES):
        np.testing.assert_allclose(got, ref, rtol=2e-2, atol=5e-2, err_msg=key)


def bf16_data(case, seed):
    B, H, T, nh, dk, dv, chunk = case
    d = make(B, H, T, nh, dk, dv, seed=seed)
    rnd = lambda x: torch.as_tensor(x, dtype=torch.float32).to(torch.bfloat16).double().numpy()
    for k in ("Q", "K", "V", "beta", "grad_y"):
        d[k] = rnd(d[k])
    return d


# bf16 inputs run on the tensor-core kernels (d_k, d_v multiples of 8,
# nh * chunk <= 64): value-column splits of 2 (d_v > 32, few heads) and 1
# (many heads, or d_v <= 32), padded d_k / d_v / chunk rows, nh > 1, ragged T.
TC_CASES = [  # (B, H, T, nh, dk, dv, chunk)
    (1, 2, 100, 1, 64, 64, 64), (2, 1, 77, 2, 32, 32, 32), (1, 2, 130, 1, 16, 16, 16),
    (2, 2, 19, 1, 8, 8, 8), (1, 1, 65, 1, 64, 32, 64), (1, 3, 40, 4, 8, 16, 16),
    (1, 2, 90, 1, 48, 40, 64), (10, 8, 70, 1, 64, 64, 64), (1, 1, 1, 1, 8, 8, 64),
]
# The bar for bf16 inputs is rtol 2e-2 (outputs and input gradients are bf16).
# The fp32 outputs (H_T, dH0) are held to 1e-3: the split hi/lo tensor-core
# products keep the state chain fp32-grade, so a precision regression there
# shows up long before the 2e-2 bar.
BF16_TOL = dict(rtol=2e-2, atol=2e-2)
BF16_GRAD_TOL = dict(rtol=2e-2, atol=5e-2)
FP32_STATE_TOL = dict(rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("case", TC_CASES)
def test_bf16_tensor_core_vs_oracle(cuda, case):
    d = bf16_data(case, seed=sum(case) + 1)
    ry, rHT, rg = oracle_ref(d, case[-1])
    y, HT, *grads = run(d, case[-1], cuda, torch.bfloat16)
    np.testing.assert_allclose(y, ry, **BF16_TOL)
    np.testing.assert_allclose(HT, rHT, **FP32_STATE_TOL)
    for got, ref, key in zip(grads, rg, NAMES):
        tol = FP32_STATE_TOL if key == "dH0" else BF16_GRAD_TOL
        np.testing.assert_allclose(got, ref, **tol, err_msg=key)


def test_full_length_config5_bf16(cuda):
    """BASELINE config 5 per (b, h) at full length in its own dtype: bf16 Q/K/V/beta,
    fp32 state, H=8, d_k=d_v=64, chunk=64, T=8192 (B=1 for the fp64 oracle)."""
    case = (1, 8, 8192, 1, 64, 64, 64)
    d = bf16_data(case, seed=5)
    d["H0"][:] = 0.0
    ry, rHT, rg = oracle_ref(d, 64)
    y, HT, *grads = run(d, 64, cuda, torch.bfloat16)
    np.testing.assert_allclose(y, ry, **BF16_TOL)
    np.testing.assert_allclose(HT, rHT, **FP32_STATE_TOL)
    for got, ref, key in zip(grads, rg, NAMES):
        # sums over up to 8192 tokens: the absolute floor follows the gradient's magnitude
        tol = dict(BF16_GRAD_TOL)
        tol["atol"] = max(tol["atol"], 1e-3 * float(np.abs(ref).max()))
        np.testing.assert_allclose(got, ref, **tol, err_msg=key)


def test_full_length_config5_fp32(cuda):
    """BASELINE config 5 shape per (b, h) at full length: H=8, d_k=d_v=64,
    chunk=64, T=8192 (B=1 to keep the fp64 oracle quick)."""
    d = make(1, 8, 8192, 1, 64, 64, seed=0)
    d["H0"][:] = 0.0
    ry, rHT, rg = oracle_ref(d, 64)
    y, HT, *grads = run(d, 64, cuda)
    # 128 chained chunk-state updates: fp32 rounding of the state accumulates
    # along the chain, so the absolute floor is twice the short-sequence one.
    fwd_long = dict(rtol=1e-5, atol=2e-5)
    np.testing.assert_allclose(y, ry, **fwd_long)
    np.testing.assert_allclose(HT, rHT, **fwd_long)
    for got, ref, key in zip(grads, rg, NAMES):
        # gradients sum over up to 8192 tokens: the absolute floor scales with
        # the gradient's own magnitude (norm-relative 1e-5)
        tol = dict(rtol=BWD["rtol"], atol=max(BWD["atol"], 1e-5 * float(np.abs(ref).max())))
        np.testing.assert_allclose(got, ref, **tol, err_msg=key)


def test_envelope_errors(cuda):
    import mingru_b200 as mb

    Q = torch.randn(1, 1, 10, 8, device=cuda)
    K = torch.randn(1, 1, 10, 2, 8, device=cuda)
    V = torch.randn(1, 1, 10, 2, 8, device=cuda)
    b = torch.rand(1, 1, 10, 2, device=cuda)
    H0 = torch.zeros(1, 1, 8, 8, device=cuda)
    with pytest.raises(ValueError, match="envelope"):
        mb.delta_scan_impl(Q, K, V, b, H0, chunk_size=64)
    with pytest.raises(ValueError, match="disagree"):
        mb.delta_scan_impl(Q, K, V[..., :4], b, H0, chunk_size=4)
