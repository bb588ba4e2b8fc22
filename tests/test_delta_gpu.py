"""GPU parity of the DeltaMinGRU chunked-WY delta rule (fwd + bwd) against the
reference's golden vectors (DeltaMinGRU._forward_chunked through the
reference's raw-tensor shim, min_gru.py:3152-3255) and the fp64 oracle
(chunked restatement + the sequential micro-step recurrence).

Tolerances. The parity bar: fp32 forward rtol 1e-5 / atol 1e-6, gradients
rtol 1e-4 / atol 1e-5; bf16 inputs with fp32 state rtol 2e-2 / atol 2e-2
(outputs and input gradients are bf16), and the fp32 state outputs of a bf16
run (H_T, dH0) rtol 1e-3 / atol 1e-3. Where the reference's OWN eager path
deviates more between fp32 and fp64 on the same inputs (the unit-triangular
solves and the chunk-state chain round in fp32 in any implementation), the
absolute part of the tolerance is 10x that deviation -- the reference parity
runner's rule (triton_scans.py:3303-3330); the deviations come from
tests/golden/eager_dev.json, made by tests/golden/make_golden.py --eager-dev
with the reference on the same inputs (tests/cases.py). Every comparison
prints |kernel - fp64|, |eager32 - fp64| and their ratio."""

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
BF16 = dict(rtol=2e-2, atol=2e-2)
FP32_STATE = dict(rtol=1e-3, atol=1e-3)

EAGER_DEV = json.loads((GOLDEN / "eager_dev.json").read_text())


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
    mb.raise_device_error(dev)
    out = {"y": f64(y), "H_T": f64(HT)}
    out.update(zip(C.DELTA_NAMES, (f64(Q.grad), f64(K.grad), f64(V.grad), f64(beta.grad),
                                   f64(H0.grad))))
    return out


def oracle_ref(d, chunk):
    y, HT = delta_oracle.delta_forward(d["Q"], d["K"], d["V"], d["beta"], d["H0"], chunk)
    grads = delta_oracle.delta_backward(d["Q"], d["K"], d["V"], d["beta"], d["H0"],
                                        d["grad_y"], d["grad_H_T"], chunk)
    out = {"y": y, "H_T": HT}
    out.update(zip(C.DELTA_NAMES, grads))
    return out


def compare(label, got, ref, bars, dev):
    """Check every tensor against `ref` under its gate; print the deviations."""
    for name in ["y", "H_T"] + C.DELTA_NAMES:
        print(C.report(label, got[name], ref[name], dev, name))
    for name in ["y", "H_T"] + C.DELTA_NAMES:
        np.testing.assert_allclose(got[name], ref[name], **C.gate(bars[name], dev, name),
                                   err_msg=f"{label} {name}")


FP32_BARS = {"y": FWD, "H_T": FWD, **{k: BWD for k in C.DELTA_NAMES}}
BF16_BARS = {"y": BF16, "H_T": FP32_STATE, "dQ": BF16, "dK": BF16, "dV": BF16, "dbeta": BF16,
             "dH0": FP32_STATE}


@pytest.mark.parametrize("name", golden_names("delta_"))
def test_golden(cuda, name):
    g = load_golden(name)
    got = run(g, int(g["chunk"]), cuda)
    ref = {"y": g["y"], "H_T": g["H_T"], **{k: g[k] for k in C.DELTA_NAMES}}
    compare(name, got, ref, FP32_BARS, EAGER_DEV["golden:" + name])


@pytest.mark.parametrize("case", C.DELTA_CASES)
def test_vs_oracle(cuda, case):
    d = C.delta_case_inputs("fp32", case)
    compare(str(case), run(d, case[-1], cuda), oracle_ref(d, case[-1]), FP32_BARS,
            EAGER_DEV[C.case_key("delta_fp32", case)])


@pytest.mark.parametrize("case", C.DELTA_TC_CASES)
def test_bf16_tensor_core_vs_oracle(cuda, case):
    """bf16 inputs (tensor-core kernels) against the fp64 oracle on the
    bf16-rounded inputs."""
    d = C.delta_case_inputs("bf16", case)
    compare(str(case), run(d, case[-1], cuda, torch.bfloat16), oracle_ref(d, case[-1]), BF16_BARS,
            EAGER_DEV[C.case_key("delta_bf16", case)])


FP16 = dict(rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("case", [(1, 2, 100, 1, 64, 64, 64), (2, 1, 77, 2, 32, 32, 32),
                                  (1, 1, 70, 1, 128, 128, 64)])
def test_fp16_inputs_vs_oracle(cuda, case):
    """fp16 inputs: fp32 arithmetic (the fp32 kernels), outputs and input
    gradients rounded once to fp16 (relative 2^-11), against the fp64 oracle on
    the fp16-rounded inputs."""
    d = C.delta_case_inputs("fp32", case)
    for k in ("Q", "K", "V", "beta", "grad_y"):
        d[k] = d[k].astype(np.float16).astype(np.float64)
    got = run(d, case[-1], cuda, torch.float16)
    ref = oracle_ref(d, case[-1])
    bars = {"y": FP16, "H_T": FWD, "dQ": FP16, "dK": FP16, "dV": FP16, "dbeta": FP16,
            "dH0": BWD}
    dev = EAGER_DEV[C.case_key("delta_fp32", case)]  # the fp32 states: fp32 gates
    for name in ["y", "H_T"] + C.DELTA_NAMES:
        print(C.report(str(case), got[name], ref[name], dev, name))
        if bars[name] is FP16:  # one fp16 rounding of values up to max|ref|
            tol = dict(rtol=FP16["rtol"], atol=FP16["atol"] * max(1.0, float(np.max(np.abs(ref[name])))))
        else:
            tol = C.gate(bars[name], dev, name)
        np.testing.assert_allclose(got[name], ref[name], **tol, err_msg=f"{case} {name}")


def test_full_length_config5_bf16(cuda):
    """BASELINE config 5 at full size in its own dtype: bf16 Q/K/V/beta, fp32
    state, B=8, H=8, d_k=d_v=64, chunk=64, T=8192."""
    d = C.delta_full_inputs(bf16=True)
    compare("config5 bf16", run(d, 64, cuda, torch.bfloat16), oracle_ref(d, 64), BF16_BARS,
            EAGER_DEV["delta_full_bf16"])


def test_full_length_config5_fp32(cuda):
    """BASELINE config 5 shape at full size with fp32 inputs: B=8, H=8,
    d_k=d_v=64, chunk=64, T=8192."""
    d = C.delta_full_inputs(bf16=False)
    compare("config5 fp32", run(d, 64, cuda), oracle_ref(d, 64), FP32_BARS,
            EAGER_DEV["delta_full_fp32"])


def test_envelope_errors(cuda):
    import mingru_b200 as mb

    def args(T, nh, dk, dv):
        return (torch.randn(1, 1, T, dk, device=cuda), torch.randn(1, 1, T, nh, dk, device=cuda),
                torch.randn(1, 1, T, nh, dv, device=cuda), torch.rand(1, 1, T, nh, device=cuda),
                torch.zeros(1, 1, dk, dv, device=cuda))

    with pytest.raises(ValueError, match="envelope"):  # d_k above 128
        mb.delta_scan_impl(*args(10, 1, 136, 8), chunk_size=16)
    with pytest.raises(ValueError, match="envelope"):  # one token's micro-steps do not fit
        mb.delta_scan_impl(*args(10, 200, 64, 64), chunk_size=1)
    Q, K, V, b, H0 = args(10, 2, 8, 8)
    with pytest.raises(ValueError, match="disagree"):
        mb.delta_scan_impl(Q, K, V[..., :4], b, H0, chunk_size=4)
