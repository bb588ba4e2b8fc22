"""GPU parity of matrix_scan / matrix_affine_scan (fwd + bwd) against the
reference's golden vectors and the fp64 oracle (sequential restatement of
min_gru.py:1513-1655 and the adjoint of triton_scans.py:823-959).

Tolerances: fp32 forward rtol 1e-5 / atol 1e-6 and gradients rtol 1e-4 /
atol 1e-5 against fp64; bf16 inputs with fp32 state rtol 2e-2."""

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


def run_affine(A, Bm, gA, gB, dev, dtype=torch.float32):
    import mingru_b200 as mb

    tA = torch.as_tensor(A, dtype=dtype, device=dev).requires_grad_(True)
    tB = torch.as_tensor(Bm, dtype=dtype, device=dev).requires_grad_(True)
    Ab, Bb = mb.matrix_affine_scan(tA, tB)
    torch.autograd.backward([Ab, Bb], [torch.as_tensor(gA, dtype=dtype, device=dev),
                                       torch.as_tensor(gB, dtype=dtype, device=dev)])
    mb.raise_device_error(dev)
    return f64(Ab), f64(Bb), f64(tA.grad), f64(tB.grad)


@pytest.mark.parametrize("name", golden_names("affine_"))
def test_affine_golden(cuda, name):
    g = load_golden(name)
    Ab, Bb, dA, dB = run_affine(g["A"], g["Bm"], g["gAbar"], g["gBbar"], cuda)
    np.testing.assert_allclose(Ab, g["Abar"], **FWD)
    np.testing.assert_allclose(Bb, g["Bbar"], **FWD)
    np.testing.assert_allclose(dA, g["dA"], **BWD)
    np.testing.assert_allclose(dB, g["dBm"], **BWD)


@pytest.mark.parametrize("name", golden_names("matrix_"))
def test_matrix_golden(cuda, name):
    import mingru_b200 as mb

    g = load_golden(name)
    M = torch.as_tensor(g["M"], dtype=torch.float32, device=cuda).requires_grad_(True)
    b = torch.as_tensor(g["b"], dtype=torch.float32, device=cuda).requires_grad_(True)
    A, Bc = mb.matrix_scan(M, b)
    assert A.shape == M.shape and Bc.shape == b.shape
    torch.autograd.backward([A, Bc], [torch.as_tensor(g["gA"], dtype=torch.float32, device=cuda),
                                      torch.as_tensor(g["gBc"], dtype=torch.float32, device=cuda)])
    np.testing.assert_allclose(f64(A), g["A"], **FWD)
    np.testing.assert_allclose(f64(Bc), g["Bc"], **FWD)
    np.testing.assert_allclose(f64(M.grad), g["dM"], **BWD)
    np.testing.assert_allclose(f64(b.grad), g["db"], **BWD)


def contractive_inputs(B, T, n, k, v, seed):
    """The reference parity harness's generator (triton_scans.py:2682-2690):
    A ~ N(0,1) * 0.5 / sqrt(k) keeps the running product bounded."""
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((B, T, n, k, k)) * (0.5 / math.sqrt(k))
    Bm = rng.standard_normal((B, T, n, k, v))
    gA = rng.standard_normal((B, T, n, k, k))
    gB = rng.standard_normal((B, T, n, k, v))
    return [x.astype(np.float32).astype(np.float64) for x in (A, Bm, gA, gB)]


CASES = [(2, 13, 3, 2, 1), (1, 64, 33, 2, 1), (2, 100, 40, 1, 1), (2, 50, 5, 1, 4),
         (1, 70, 9, 2, 4), (2, 33, 7, 4, 1), (1, 40, 35, 4, 2), (1, 37, 3, 4, 8),
         (2, 29, 33, 8, 1), (1, 20, 3, 8, 2), (1, 12, 2, 16, 1), (1, 9, 3, 5, 1),
         (2, 11, 2, 3, 2), (1, 300, 64, 2, 16), (3, 1, 4, 2, 1)]


@pytest.mark.parametrize("case", CASES)
def test_affine_vs_oracle(cuda, case):
    A, Bm, gA, gB = contractive_inputs(*case, seed=sum(case))
    rA, rB = oracle.matrix_affine_scan(A, Bm)
    rdA, rdB = oracle.matrix_affine_scan_bwd(A, rA, rB, gA, gB)
    Ab, Bb, dA, dB = run_affine(A, Bm, gA, gB, cuda)
    np.testing.assert_allclose(Ab, rA, **FWD)
    np.testing.assert_allclose(Bb, rB, **FWD)
    np.testing.assert_allclose(dA, rdA, **BWD)
    np.testing.assert_allclose(dB, rdB, **BWD)


# Shapes that take the TMA strip path (k (k+v) <= 8, >= ~3/4 of the SMs'
# worth of 32-block strips): a ragged T and a partial last strip (n = 250),
# k = 1, and v = 2.
STRIP_CASES = [(14, 77, 250, 2, 1), (4, 100, 1024, 1, 1), (8, 65, 512, 2, 2)]


@pytest.mark.parametrize("case", STRIP_CASES)
def test_affine_strip_path_vs_oracle(cuda, case):
    A, Bm, gA, gB = contractive_inputs(*case, seed=sum(case))
    rA, rB = oracle.matrix_affine_scan(A, Bm)
    rdA, rdB = oracle.matrix_affine_scan_bwd(A, rA, rB, gA, gB)
    Ab, Bb, dA, dB = run_affine(A, Bm, gA, gB, cuda)
    np.testing.assert_allclose(Ab, rA, **FWD)
    np.testing.assert_allclose(Bb, rB, **FWD)
    np.testing.assert_allclose(dA, rdA, **BWD)
    np.testing.assert_allclose(dB, rdB, **BWD)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", [(2, 40, 33, 2, 1), (1, 20, 9, 8, 1), (16, 96, 256, 2, 1)])
def test_affine_half_inputs(cuda, case, dtype):
    A, Bm, gA, gB = contractive_inputs(*case, seed=3)
    rnd = lambda x: torch.as_tensor(x, dtype=torch.float32).to(dtype).double().numpy()
    A, Bm, gA, gB = rnd(A), rnd(Bm), rnd(gA), rnd(gB)
    rA, rB = oracle.matrix_affine_scan(A, Bm)
    rdA, rdB = oracle.matrix_affine_scan_bwd(A, rA, rB, gA, gB)
    Ab, Bb, dA, dB = run_affine(A, Bm, gA, gB, cuda, dtype)
    tol = dict(rtol=2e-2, atol=2e-2)
    for got, ref in ((Ab, rA), (Bb, rB), (dA, rdA), (dB, rdB)):
        np.testing.assert_allclose(got, ref, **tol)


def test_reference_identities(cuda):
    """k=2/v=1 matrix_affine_scan == matrix_scan, and identity transitions
    accumulate the inputs (test_scan_ops.py:239-245, 280-288)."""
    import mingru_b200 as mb

    g = torch.Generator().manual_seed(42)
    M = (torch.randn(2, 50, 3, 2, 2, generator=g) * 0.3).to(cuda)
    b = torch.randn(2, 50, 3, 2, generator=g).to(cuda)
    A1, B1 = mb.matrix_scan(M, b)
    A2, B2 = mb.matrix_affine_scan(M, b.unsqueeze(-1))
    assert torch.equal(A1, A2) and torch.equal(B1, B2.squeeze(-1))
    eye = torch.eye(2, device=cuda).expand(2, 50, 3, 2, 2).contiguous()
    _, Bc = mb.matrix_scan(eye, b)
    torch.testing.assert_close(Bc, torch.cumsum(b, 1), rtol=1e-5, atol=1e-5)


def test_envelope_errors(cuda):
    import mingru_b200 as mb

    A = torch.randn(2, 5, 3, 4, 4, device=cuda)
    with pytest.raises(ValueError, match="k rows"):
        mb.matrix_affine_scan(A, torch.randn(2, 5, 3, 3, 1, device=cuda))
    with pytest.raises(ValueError, match="5-D"):
        mb.matrix_affine_scan(A[0], torch.randn(5, 3, 4, 1, device=cuda))
    with pytest.raises(ValueError, match=r"\(B, T, n, 2, 2\)"):
        mb.matrix_scan(A, torch.randn(2, 5, 3, 2, device=cuda))


def test_full_config3_fp32(cuda):
    """BASELINE config 3 at full size: B=16, T=2048, n=256 (D=512) 2x2 blocks,
    M = sigmoid(N(0,1)) * R(theta), theta ~ U(-pi, pi), b ~ N(0,1)."""
    B, T, n = 16, 2048, 256
    g = torch.Generator().manual_seed(0)
    th = (torch.rand(B, T, n, generator=g) * 2 - 1) * math.pi
    s = torch.sigmoid(torch.randn(B, T, n, generator=g))
    c, sn = torch.cos(th), torch.sin(th)
    M = s[..., None, None] * torch.stack([torch.stack([c, -sn], -1), torch.stack([sn, c], -1)], -2)
    b = torch.randn(B, T, n, 2, generator=g)
    gA = torch.zeros(B, T, n, 2, 2)
    gB = torch.randn(B, T, n, 2, generator=torch.Generator().manual_seed(1234))
    rA, rB = oracle.matrix_scan(M.numpy(), b.numpy())
    rdM, rdb = oracle.matrix_scan_bwd(M.numpy(), rA, rB, gA.numpy(), gB.numpy())
    Ab, Bb, dA, dB = run_affine(M, b.unsqueeze(-1), gA, gB.unsqueeze(-1), cuda)
    np.testing.assert_allclose(Ab, rA, **FWD)
    np.testing.assert_allclose(Bb[..., 0], rB, **FWD)
    np.testing.assert_allclose(dA, rdM, **BWD)
    np.testing.assert_allclose(dB[..., 0], rdb, **BWD)
