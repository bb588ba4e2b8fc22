"""GPU parity of parallel_scan_log (fwd + bwd) against the reference's golden
vectors and the fp64 oracle (sequential restatement of min_gru.py:755-807).

Tolerances: fp32 forward rtol 1e-5 / atol 1e-6 and gradients rtol 1e-4 /
atol 1e-5, both against fp64. (The reference's own fp32 eager path is NOT
within these bounds of fp64 at long T -- its global cumsum of log
coefficients cancels ~T ulps -- so fp64 is the stricter oracle.) bf16 /
fp16 inputs with fp32 state: rtol 2e-2 against fp64 on the rounded inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from oracle import oracle

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
BWD = dict(rtol=1e-4, atol=1e-5)


def softplus(x):
    return np.logaddexp(0.0, x)


def log_space_inputs(B, T, D, seed, h0_scale=0.1):
    """MinGRU's construction (min_gru.py:1383-1397): lc = -softplus(k),
    lv = [log h0, -softplus(-k) + log_g(x)] with k, x ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((B, T, D))
    x = rng.standard_normal((B, T, D))
    log_g = np.where(x >= 0, np.log(np.maximum(x, 0) + 0.5), -softplus(-x))
    lc = -softplus(k)
    lv = np.concatenate([rng.standard_normal((B, 1, D)) * h0_scale, -softplus(-k) + log_g], 1)
    gh = rng.standard_normal((B, T, D))
    return lc, lv, gh


def run(lc, lv, gh, dev, dtype=torch.float32):
    import mingru_b200 as mb

    tlc = torch.as_tensor(lc, dtype=dtype, device=dev).requires_grad_(True)
    tlv = torch.as_tensor(lv, dtype=dtype, device=dev).requires_grad_(True)
    h = mb.parallel_scan_log(tlc, tlv)
    h.backward(torch.as_tensor(gh, dtype=dtype, device=dev))
    mb.raise_device_error(dev)
    f = lambda t: t.detach().float().cpu().numpy().astype(np.float64)
    return f(h), f(tlc.grad), f(tlv.grad)


@pytest.mark.parametrize("name", golden_names("log_"))
def test_golden(cuda, name):
    g = load_golden(name)
    h, dlc, dlv = run(g["log_coeffs"], g["log_values"], g["grad_h"], cuda)
    np.testing.assert_allclose(h, g["h"], **FWD)
    np.testing.assert_allclose(dlc, g["dlog_coeffs"], **BWD)
    np.testing.assert_allclose(dlv, g["dlog_values"], **BWD)


# Paths (B200, 148 SMs): column path when T <= 1024, D*size % 16 == 0 and
# B*ceil(D/8) >= 148 (whole time axis per CTA), with 16-channel CTAs when
# B*ceil(D/16) >= 111 ((3, 100, 1000), (40, 77, 36) with a 4-channel tail,
# (150, 5, 8) with T < 32) and 8-channel CTAs otherwise ((19, 1024, 64),
# (2, 1024, 600)); strip path for longer T with >= 296 32-channel strips
# ((10, 1500, 960)); direct tiles otherwise.
SHAPES = [(1, 1, 1), (2, 13, 3), (3, 31, 4), (2, 33, 129), (1, 64, 256), (3, 100, 1000),
          (2, 1000, 36), (2, 50, 40), (10, 100, 1000), (3, 70, 3200),
          (40, 77, 36), (150, 5, 8), (19, 1024, 64), (37, 1000, 40), (2, 1024, 600),
          (10, 1500, 960), (3, 1100, 200)]


@pytest.mark.parametrize("shape", SHAPES)
def test_vs_oracle_fp32(cuda, shape):
    lc, lv, gh = log_space_inputs(*shape, seed=sum(shape))
    lc, lv, gh = (x.astype(np.float32).astype(np.float64) for x in (lc, lv, gh))
    rh = oracle.parallel_scan_log(lc, lv)
    rdlc, rdlv = oracle.parallel_scan_log_bwd(lc, lv, gh)
    h, dlc, dlv = run(lc, lv, gh, cuda)
    np.testing.assert_allclose(h, rh, **FWD)
    np.testing.assert_allclose(dlc, rdlc, **BWD)
    np.testing.assert_allclose(dlv, rdlv, **BWD)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 13, 3), (2, 300, 256), (10, 45, 1000), (40, 77, 64),
                                   (2, 300, 600), (10, 1500, 960)])
def test_half_inputs_fp32_state(cuda, shape, dtype):
    lc, lv, gh = log_space_inputs(*shape, seed=5)
    rnd = lambda x: torch.as_tensor(x, dtype=torch.float32).to(dtype).double().numpy()
    lc, lv, gh = rnd(lc), rnd(lv), rnd(gh)
    rh = oracle.parallel_scan_log(lc, lv)
    rdlc, rdlv = oracle.parallel_scan_log_bwd(lc, lv, gh)
    h, dlc, dlv = run(lc, lv, gh, cuda, dtype)
    tol = dict(rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(h, rh, **tol)
    np.testing.assert_allclose(dlc, rdlc, **tol)
    np.testing.assert_allclose(dlv, rdlv, **tol)


@pytest.mark.parametrize("shape", [(2, 40, 8), (40, 40, 36)])
def test_zero_initial_state_and_empty(cuda, shape):
    import mingru_b200 as mb

    lc, lv, gh = log_space_inputs(*shape, seed=3)
    lv[:, 0] = np.log(np.finfo(np.float32).tiny)  # h0 numerically zero
    rh = oracle.parallel_scan_log(lc, lv)
    h, _, _ = run(lc, lv, gh, cuda)
    np.testing.assert_allclose(h, rh, **FWD)
    lv[:, 0] = -np.inf  # exact zero initial state
    rh = oracle.parallel_scan_log(lc, lv)
    h, dlc, dlv = run(lc, lv, gh, cuda)
    np.testing.assert_allclose(h, rh, **FWD)
    assert np.all(dlv[:, 0] == 0)
    lc0 = torch.zeros(2, 0, 5, device=cuda, requires_grad=True)
    lv0 = torch.zeros(2, 1, 5, device=cuda, requires_grad=True)
    h0 = mb.parallel_scan_log(lc0, lv0)
    assert h0.shape == (2, 0, 5)
    h0.sum().backward()
    assert torch.all(lv0.grad == 0)


def test_full_config1_fp32(cuda):
    """BASELINE config 1 at full size (B=8, T=1024, D=256), log h0 = log(tiny)."""
    lc, lv, gh = log_space_inputs(8, 1024, 256, seed=0)
    lv[:, 0] = np.log(np.finfo(np.float32).tiny)
    lc, lv, gh = (x.astype(np.float32).astype(np.float64) for x in (lc, lv, gh))
    rh = oracle.parallel_scan_log(lc, lv)
    rdlc, rdlv = oracle.parallel_scan_log_bwd(lc, lv, gh)
    h, dlc, dlv = run(lc, lv, gh, cuda)
    np.testing.assert_allclose(h, rh, **FWD)
    np.testing.assert_allclose(dlc, rdlc, **BWD)
    np.testing.assert_allclose(dlv, rdlv, **BWD)


@pytest.mark.parametrize("case", ["positive_log_coeff", "tiny_log_values", "large_log_values",
                                  "large_h0", "mixed"])
@pytest.mark.parametrize("B", [40, 19])  # 16- and 8-channel column CTAs
def test_column_path_log_space_fallback(cuda, case, B):
    """Column-path CTAs whose data leaves the linear-domain envelope (a log
    coefficient > 0, a log value outside [-30, 20], or log h_0 > 20) run the log-space
    monoid; the other CTAs of the same launch stay linear."""
    T, D = 200, 64  # B*8 >= 148 column groups: column path
    lc, lv, gh = log_space_inputs(B, T, D, seed=11)
    if case in ("positive_log_coeff", "mixed"):
        lc[3, 50:60, 9] = 0.05  # a_t > 1 in one channel of one group
    if case in ("tiny_log_values", "mixed"):
        lv[7, 1:120, 17] -= 40.0  # b_t ~ e^-40 for a stretch
    if case == "large_log_values":
        lv[5, 30:40, 40] += 24.0  # b_t ~ e^24
    if case == "large_h0":
        lv[2, 0, 3] = 25.0  # h_0 = e^25
    lc, lv, gh = (x.astype(np.float32).astype(np.float64) for x in (lc, lv, gh))
    rh = oracle.parallel_scan_log(lc, lv)
    rdlc, rdlv = oracle.parallel_scan_log_bwd(lc, lv, gh)
    h, dlc, dlv = run(lc, lv, gh, cuda)
    np.testing.assert_allclose(h, rh, **FWD)
    np.testing.assert_allclose(dlc, rdlc, **BWD)
    np.testing.assert_allclose(dlv, rdlv, **BWD)
