"""GPU parity of linear_scan (fwd + bwd) against the reference's golden
vectors and the fp64 oracle (sequential restatement of min_gru.py:1454-1510).

Tolerances (from the parity bar for this path): fp32 forward rtol 1e-5 /
atol 1e-6, gradients rtol 1e-4 (atol 1e-5); bf16 inputs with fp32 state
rtol 2e-2 against the fp64 oracle run on the bf16-rounded inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import oracle

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


def run(a, b, gA, gB, dev, dtype=torch.float32):
    import mingru_b200 as mb

    ta = torch.as_tensor(a, dtype=dtype, device=dev).requires_grad_(True)
    tb = torch.as_tensor(b, dtype=dtype, device=dev).requires_grad_(True)
    A, Bc = mb.linear_scan(ta, tb)
    torch.autograd.backward([A, Bc], [torch.as_tensor(gA, dtype=dtype, device=dev),
                                      torch.as_tensor(gB, dtype=dtype, device=dev)])
    mb.raise_device_error(dev)
    f = lambda t: t.detach().float().cpu().numpy().astype(np.float64)
    return f(A), f(Bc), f(ta.grad), f(tb.grad)


@pytest.mark.parametrize("name", golden_names("linear_"))
def test_golden(cuda, name):
    g = load_golden(name)
    A, Bc, da, db = run(g["a"], g["b"], g["gA"], g["gBc"], cuda)
    np.testing.assert_allclose(A, g["A"], **FWD)
    np.testing.assert_allclose(Bc, g["Bc"], **FWD)
    np.testing.assert_allclose(da, g["da"], **BWD)
    np.testing.assert_allclose(db, g["db"], **BWD)


# Strip path (B*ceil(D/32) >= 296 on 148 SMs): (10, 100, 1000) and (3, 70, 3200)
# with ragged T and a partial last strip, (19, 1100, 520) with a long ragged
# walk, (20, 300, 1000) with more strips (640) than warps in flight, so warps
# walk a second strip on the same ring. 16-bit inputs take the same strip path:
# (10, 45, 1000) and (15, 70, 1048) end in partial strips (8 and 24 channels),
# (20, 300, 1000) has 640 strips for 592 warps.
SHAPES = [(1, 1, 1), (2, 13, 3), (3, 31, 4), (2, 32, 128), (2, 33, 129), (1, 64, 256),
          (3, 100, 1000), (2, 1000, 36), (1, 777, 8), (4, 257, 512), (2, 50, 40), (1, 3000, 132),
          (10, 100, 1000), (3, 70, 3200), (19, 1100, 520), (20, 300, 1000)]


def inputs(B, T, D, seed):
    rng = np.random.default_rng(seed)
    a = np.tanh(rng.standard_normal((B, T, D)))
    b = rng.standard_normal((B, T, D))
    gA = rng.standard_normal((B, T, D))
    gB = rng.standard_normal((B, T, D))
    return a, b, gA, gB


@pytest.mark.parametrize("shape", SHAPES)
def test_vs_oracle_fp32(cuda, shape):
    a, b, gA, gB = inputs(*shape, seed=sum(shape))
    a32, b32 = a.astype(np.float32), b.astype(np.float32)
    rA, rB = oracle.linear_scan(a32, b32)
    rda, rdb = oracle.linear_scan_bwd(a32, rA, rB, gA.astype(np.float32), gB.astype(np.float32))
    A, Bc, da, db = run(a32, b32, gA.astype(np.float32), gB.astype(np.float32), cuda)
    np.testing.assert_allclose(A, rA, **FWD)
    np.testing.assert_allclose(Bc, rB, **FWD)
    np.testing.assert_allclose(da, rda, **BWD)
    np.testing.assert_allclose(db, rdb, **BWD)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 13, 3), (2, 300, 256), (3, 100, 1000), (2, 77, 40), (1, 500, 36), (10, 45, 1000),
                                   (20, 300, 1000), (15, 70, 1048)])
def test_half_inputs_fp32_state(cuda, shape, dtype):
    a, b, gA, gB = inputs(*shape, seed=7)
    rnd = lambda x: torch.as_tensor(x, dtype=torch.float32).to(dtype).double().numpy()
    a, b, gA, gB = rnd(a), rnd(b), rnd(gA), rnd(gB)
    rA, rB = oracle.linear_scan(a, b)
    rda, rdb = oracle.linear_scan_bwd(a, rA, rB, gA, gB)
    A, Bc, da, db = run(a, b, gA, gB, cuda, dtype)
    tol = dict(rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(A, rA, **tol)
    np.testing.assert_allclose(Bc, rB, **tol)
    np.testing.assert_allclose(da, rda, **tol)
    np.testing.assert_allclose(db, rdb, **tol)


def test_empty_and_noncontiguous(cuda):
    import mingru_b200 as mb

    z = torch.zeros(2, 0, 5, device=cuda)
    A, Bc = mb.linear_scan(z, z)
    assert A.shape == (2, 0, 5) and Bc.shape == (2, 0, 5)
    a = torch.rand(5, 40, 2, device=cuda).transpose(0, 2)  # (2, 40, 5), non-contiguous
    b = torch.rand(2, 40, 5, device=cuda)
    A, Bc = mb.linear_scan(a, b)
    rA, rB = oracle.linear_scan(a.cpu().double().numpy(), b.cpu().double().numpy())
    np.testing.assert_allclose(Bc.cpu().double().numpy(), rB, **FWD)
    # misaligned storage offset: still correct (the op re-packs)
    buf = torch.rand(1 + 2 * 40 * 8, device=cuda)
    a2 = buf[1:].view(2, 40, 8)
    A2, B2 = mb.linear_scan(a2, a2)
    rA2, rB2 = oracle.linear_scan(a2.cpu().double().numpy(), a2.cpu().double().numpy())
    np.testing.assert_allclose(B2.cpu().double().numpy(), rB2, **FWD)


def test_full_config2_fp32(cuda):
    """BASELINE config 2 at full size (B=16, T=4096, D=1024) against the oracle."""
    B, T, D = 16, 4096, 1024
    g = torch.Generator().manual_seed(0)
    a = torch.tanh(torch.randn(B, T, D, generator=g))
    b = torch.randn(B, T, D, generator=g)
    gB = torch.randn(B, T, D, generator=torch.Generator().manual_seed(1234))
    gA = torch.zeros(B, T, D)
    rA, rB = oracle.linear_scan(a.numpy(), b.numpy())
    rda, rdb = oracle.linear_scan_bwd(a.numpy(), rA, rB, gA.numpy(), gB.numpy())
    A, Bc, da, db = run(a, b, gA, gB, cuda)
    np.testing.assert_allclose(Bc, rB, **FWD)
    np.testing.assert_allclose(A, rA, **FWD)
    np.testing.assert_allclose(db, rdb, **BWD)
    np.testing.assert_allclose(da, rda, **BWD)


def test_full_config2_bf16(cuda):
    """BASELINE config 2 at full size with bf16 inputs and fp32 state (B=16,
    T=4096, D=1024): the 16-bit strip kernels against the fp64 oracle on the
    bf16-rounded inputs, at the bf16 bar (rtol 2e-2 / atol 2e-2)."""
    B, T, D = 16, 4096, 1024
    g = torch.Generator().manual_seed(0)
    a = torch.tanh(torch.randn(B, T, D, generator=g)).to(torch.bfloat16)
    b = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
    gB = torch.randn(B, T, D, generator=torch.Generator().manual_seed(1234)).to(torch.bfloat16)
    gA = torch.zeros(B, T, D, dtype=torch.bfloat16)
    a64, b64, gA64, gB64 = (x.double().numpy() for x in (a, b, gA, gB))
    rA, rB = oracle.linear_scan(a64, b64)
    rda, rdb = oracle.linear_scan_bwd(a64, rA, rB, gA64, gB64)
    A, Bc, da, db = run(a, b, gA, gB, cuda, torch.bfloat16)
    tol = dict(rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(Bc, rB, **tol)
    np.testing.assert_allclose(A, rA, **tol)
    np.testing.assert_allclose(db, rdb, **tol)
    np.testing.assert_allclose(da, rda, **tol)
