"""Generate the golden input/output vectors that pin the oracle and the kernels.

Runs the REFERENCE implementation (chris-santiago/minGRU, package ``mingru``
0.2.1) on its eager path (``MINGRU_SCAN=eager``) in float64 on the CPU, for
small seeded cases of every op on the scan hot path, and writes one ``.npz``
per case next to this script. It needs the reference source tree (pass
``--ref /path/to/minGRU/src``); the fixtures it writes are committed, so the
tests and the GPU box never need the reference itself.

Cases and the reference code each one exercises:
  log_*      parallel_scan_log            min_gru.py:755-807 (+ autograd)
  linear_*   linear_scan                  min_gru.py:1454-1510
  matrix_*   matrix_scan (k=2, v=1)       min_gru.py:1513-1581
  affine_*   matrix_affine_scan (k, v)    min_gru.py:1584-1655
  givens_* / rotation_*
             angle-fused path maths: M built by GivensMinGRU._coeffs /
             RotationMinGRU._coeffs (min_gru.py:2552-2602, 2137-2155) with an
             explicit decay gamma, scanned by matrix_affine_scan / matrix_scan
             and applied to h0 as in GivensMinGRU.forward (min_gru.py:2641-2647)
  delta_*    DeltaMinGRU._forward_chunked (min_gru.py:3152-3255) through the
             raw-tensor shim the reference's own parity harness uses
             (triton_scans.py:3383-3451)
  module_*   whole reference modules (MinGRU ... MinGRUStack, min_gru.py:1213-4336)
             built with a seed: constructor kwargs, state_dict, input, output
             and the gradients w.r.t. the input and every parameter
Every case stores the inputs, the outputs and the gradients of
``sum(out * cotangent)`` w.r.t. every input, with a seeded cotangent.

``--eager-dev`` instead writes ``eager_dev.json``: for the delta and angle
test cases (inputs from ``tests/cases.py``, the same functions the GPU tests
call) and their golden fixtures, the largest |eager fp32 - eager fp64|
deviation of every output and gradient of the reference's own eager path.
The GPU tests widen a tolerance's absolute part to 10x that deviation where
it exceeds the parity bar -- the reference parity runner's rule
(triton_scans.py:3303-3330). The delta path runs DeltaMinGRU._forward_chunked
(min_gru.py:3152-3255); the angle path builds each step's k x k matrix from
the plane angles (the product of the rounds' rotations, times gamma, times
diag(1, scale) for k = 2: GivensMinGRU._coeffs / RotationMinGRU._coeffs,
min_gru.py:2552-2602, 2137-2155) and scans it with matrix_affine_scan.
"""

from __future__ import annotations

import argparse
import math
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _np(t):
    return t.detach().cpu().numpy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path to the reference's src/ directory")
    ap.add_argument("--eager-dev", action="store_true",
                    help="write eager_dev.json only (the golden .npz files are left as they are)")
    ap.add_argument("--only", default=None,
                    help="comma-separated fixture names: write only these (others are left as they are)")
    args = ap.parse_args()
    only = None if args.only is None else set(args.only.split(","))
    if args.eager_dev:
        eager_dev(args.ref)
        return
    os.environ["MINGRU_SCAN"] = "eager"
    sys.path.insert(0, args.ref)
    import torch
    import torch.nn as nn
    import torch.nn.functional as F
    from mingru import min_gru as mg

    torch.set_default_dtype(torch.float64)
    dt = torch.float64

    def save(name, **arrays):
        if only is None or name in only:
            np.savez_compressed(HERE / f"{name}.npz", **{k: _np(v) for k, v in arrays.items()})

    def grads(outs, ins, seed):
        g = torch.Generator().manual_seed(seed)
        cots = [torch.randn(o.shape, generator=g, dtype=dt) for o in outs]
        total = sum((o * c).sum() for o, c in zip(outs, cots))
        gs = torch.autograd.grad(total, ins, allow_unused=True)
        return cots, [torch.zeros_like(x) if gg is None else gg for x, gg in zip(ins, gs)]

    # ---------------------------------------------------------------- log
    for name, (B, T, D) in {"log_small": (2, 7, 5), "log_t1": (2, 1, 3), "log_mid": (3, 70, 9)}.items():
        g = torch.Generator().manual_seed(11)
        k = torch.randn(B, T, D, generator=g, dtype=dt)
        x = torch.randn(B, T, D, generator=g, dtype=dt)
        lc = (-F.softplus(k)).requires_grad_(True)
        lv = torch.cat(
            [torch.randn(B, 1, D, generator=g, dtype=dt) * 0.1, -F.softplus(-k) + mg.log_g(x)], 1
        ).detach().requires_grad_(True)
        h = mg.parallel_scan_log(lc, lv)
        (gh,), (dlc, dlv) = grads([h], [lc, lv], 1234)
        save(name, log_coeffs=lc, log_values=lv, h=h, grad_h=gh, dlog_coeffs=dlc, dlog_values=dlv)

    # ------------------------------------------------------------- linear
    for name, (B, T, D) in {"linear_small": (2, 6, 4), "linear_t1": (2, 1, 3),
                            "linear_mid": (2, 77, 12)}.items():
        g = torch.Generator().manual_seed(12)
        a = torch.tanh(torch.randn(B, T, D, generator=g, dtype=dt)).requires_grad_(True)
        b = torch.randn(B, T, D, generator=g, dtype=dt).requires_grad_(True)
        A, Bc = mg.linear_scan(a, b)
        (gA, gB), (da, db) = grads([A, Bc], [a, b], 1234)
        save(name, a=a, b=b, A=A, Bc=Bc, gA=gA, gBc=gB, da=da, db=db)

    # ------------------------------------------------------------- matrix
    for name, (B, T, n) in {"matrix_small": (2, 5, 3), "matrix_mid": (2, 40, 5)}.items():
        g = torch.Generator().manual_seed(13)
        th = (torch.rand(B, T, n, generator=g, dtype=dt) * 2 - 1) * math.pi
        s = torch.sigmoid(torch.randn(B, T, n, generator=g, dtype=dt))
        c, sn = torch.cos(th), torch.sin(th)
        M = (s[..., None, None] * torch.stack(
            [torch.stack([c, -sn], -1), torch.stack([sn, c], -1)], -2)).detach().requires_grad_(True)
        b = torch.randn(B, T, n, 2, generator=g, dtype=dt).requires_grad_(True)
        A, Bc = mg.matrix_scan(M, b)
        (gA, gB), (dM, db) = grads([A, Bc], [M, b], 1234)
        save(name, M=M, b=b, A=A, Bc=Bc, gA=gA, gBc=gB, dM=dM, db=db)

    # ------------------------------------------------------------- affine
    for (B, T, n, k, v) in [(2, 5, 3, 4, 2), (2, 9, 2, 8, 1), (1, 6, 2, 2, 4), (1, 5, 2, 16, 1),
                            (2, 7, 3, 1, 2), (1, 33, 2, 8, 8)]:
        name = f"affine_k{k}_v{v}"
        g = torch.Generator().manual_seed(14 + k * 7 + v)
        A = (torch.randn(B, T, n, k, k, generator=g, dtype=dt) * (0.5 / k ** 0.5)).requires_grad_(True)
        Bm = torch.randn(B, T, n, k, v, generator=g, dtype=dt).requires_grad_(True)
        Ab, Bb = mg.matrix_affine_scan(A, Bm)
        (gA, gB), (dA, dB) = grads([Ab, Bb], [A, Bm], 1234)
        save(name, A=A, Bm=Bm, Abar=Ab, Bbar=Bb, gAbar=gA, gBbar=gB, dA=dA, dBm=dB)

    # -------------------------------------------------------- angle paths
    class Const(nn.Module):
        def __init__(self, t):
            super().__init__()
            self.t = t

        def forward(self, x):
            return self.t

    for name, (B, T, in_sz, hid, blk, R, decay) in {
        "givens_k8_r3_decay": (2, 9, 4, 32, 8, 3, True),
        "givens_k8_r2": (2, 6, 4, 16, 8, 2, False),
        "givens_k4_r3_decay": (1, 7, 4, 8, 4, 3, True),
    }.items():
        torch.manual_seed(21)
        mod = mg.GivensMinGRU(in_sz, hid, block_size=blk, rounds=R).double()
        n, half = hid // blk, blk // 2
        g = torch.Generator().manual_seed(22)
        theta = ((torch.rand(B, T, n, R, half, generator=g, dtype=dt) * 2 - 1) * math.pi).requires_grad_(True)
        gamma = (torch.sigmoid(torch.randn(B, T, n, generator=g, dtype=dt)) if decay
                 else torch.ones(B, T, n, dtype=dt)).requires_grad_(True)
        bb = torch.randn(B, T, n, blk, generator=g, dtype=dt).requires_grad_(True)
        h0 = torch.randn(B, n, blk, generator=g, dtype=dt).requires_grad_(True)
        mod.linear_theta = Const(theta.reshape(B, T, n * R * half))
        M, _ = mod._coeffs(torch.zeros(B, T, in_sz, dtype=dt), None)
        M = gamma[..., None, None] * M
        Ab, Bb = mg.matrix_affine_scan(M, bb.unsqueeze(-1))
        h = torch.einsum("btnij,bnj->btni", Ab, h0) + Bb.squeeze(-1)
        perm, sgn, p2p = mod._angle_plane_meta(torch.device("cpu"))
        scale = torch.ones(B, T, n, dtype=dt)
        (gh,), (dth, dga, dbb, dh0) = grads([h], [theta, gamma, bb, h0], 1234)
        save(name, theta=theta, scale=scale, gamma=gamma, b=bb, h0=h0, perm=perm, sgn=sgn,
             p2p=p2p, h=h, grad_h=gh, dtheta=dth, dgamma=dga, db=dbb, dh0=dh0,
             flags=torch.tensor([0, int(decay)]))

    for name, (B, T, n, decay) in {"rotation_decay": (2, 8, 3, True), "rotation": (2, 5, 4, False)}.items():
        torch.manual_seed(23)
        mod = mg.RotationMinGRU(4, 2 * n, snap=None).double()
        g = torch.Generator().manual_seed(24)
        theta = ((torch.rand(B, T, n, 1, 1, generator=g, dtype=dt) * 2 - 1) * math.pi).requires_grad_(True)
        scale = torch.tanh(torch.randn(B, T, n, generator=g, dtype=dt)).requires_grad_(True)
        gamma = (torch.sigmoid(torch.randn(B, T, n, generator=g, dtype=dt)) if decay
                 else torch.ones(B, T, n, dtype=dt)).requires_grad_(True)
        bb = torch.randn(B, T, n, 2, generator=g, dtype=dt).requires_grad_(True)
        h0 = torch.randn(B, n, 2, generator=g, dtype=dt).requires_grad_(True)
        c, s = torch.cos(theta[..., 0, 0]), torch.sin(theta[..., 0, 0])
        # M = R(theta) diag(1, scale), rows as in RotationMinGRU._coeffs (min_gru.py:2146-2148)
        M = torch.stack([torch.stack([c, -s * scale], -1), torch.stack([s, c * scale], -1)], -2)
        M = gamma[..., None, None] * M
        A, Bc = mg.matrix_scan(M, bb)
        h = torch.einsum("btnij,bnj->btni", A, h0) + Bc
        perm, sgn, p2p = mod._angle_plane_meta(torch.device("cpu"))
        (gh,), (dth, dsc, dga, dbb, dh0) = grads([h], [theta, scale, gamma, bb, h0], 1234)
        save(name, theta=theta, scale=scale, gamma=gamma, b=bb, h0=h0, perm=perm, sgn=sgn,
             p2p=p2p, h=h, grad_h=gh, dtheta=dth, dscale=dsc, dgamma=dga, db=dbb, dh0=dh0,
             flags=torch.tensor([1, int(decay)]))

    # -------------------------------------------------------------- delta
    def delta_ref(Q, K, V, beta, H0, chunk):
        Bq, nH, Tq, dk = Q.shape
        nh, dv = K.shape[3], V.shape[4]
        q = Q.permute(0, 2, 1, 3)
        ks = list(K.permute(0, 2, 3, 1, 4).unbind(2))
        vs = list(V.permute(0, 2, 3, 1, 4).unbind(2))
        bs = list(beta.permute(0, 2, 3, 1).unbind(2))
        shim = types.SimpleNamespace(nh=nh, n_heads=nH, d_k=dk, d_v=dv, chunk_size=chunk,
                                     _coeffs=lambda x: (q, ks, vs, bs))
        y, HT = mg.DeltaMinGRU._forward_chunked(shim, Q.new_empty(Bq, Tq, 1), H0)
        return y.permute(0, 2, 1, 3), HT  # y back to (B, H, T, d_v)

    for name, (B, H, T, nh, dk, dv, chunk) in {
        "delta_small": (2, 2, 11, 1, 8, 8, 4),
        "delta_nh2": (1, 2, 13, 2, 4, 4, 5),
        "delta_d16": (1, 1, 40, 1, 16, 16, 16),
        "delta_c64": (1, 2, 130, 1, 32, 32, 64),
    }.items():
        g = torch.Generator().manual_seed(31)
        Q = torch.randn(B, H, T, dk, generator=g, dtype=dt).requires_grad_(True)
        K = F.normalize(torch.randn(B, H, T, nh, dk, generator=g, dtype=dt), dim=-1).requires_grad_(True)
        V = torch.randn(B, H, T, nh, dv, generator=g, dtype=dt).requires_grad_(True)
        beta = (2 * torch.sigmoid(torch.randn(B, H, T, nh, generator=g, dtype=dt))).requires_grad_(True)
        H0 = (torch.randn(B, H, dk, dv, generator=g, dtype=dt) * 0.1).requires_grad_(True)
        y, HT = delta_ref(Q, K, V, beta, H0, chunk)
        (gy, gHT), (dQ, dK, dV, dbeta, dH0) = grads([y, HT], [Q, K, V, beta, H0], 1234)
        save(name, Q=Q, K=K, V=V, beta=beta, H0=H0, y=y, H_T=HT, grad_y=gy, grad_H_T=gHT,
             dQ=dQ, dK=dK, dV=dV, dbeta=dbeta, dH0=dH0, chunk=torch.tensor(chunk))

    # ------------------------------------------------------- delta, decay
    # DeltaMinGRU._forward_chunked_gated (min_gru.py:3290-3448) through the same
    # raw-tensor shim, with lambda and dt as inputs (log gamma = -lambda dt).
    def delta_gated_ref(Q, K, V, beta, H0, lam, dtt, chunk):
        Bq, nH, Tq, dk = Q.shape
        nh, dv = K.shape[3], V.shape[4]
        q = Q.permute(0, 2, 1, 3)
        ks = list(K.permute(0, 2, 3, 1, 4).unbind(2))
        vs = list(V.permute(0, 2, 3, 1, 4).unbind(2))
        bs = list(beta.permute(0, 2, 3, 1).unbind(2))
        shim = types.SimpleNamespace(nh=nh, n_heads=nH, d_k=dk, d_v=dv, chunk_size=chunk,
                                     _coeffs=lambda x: (q, ks, vs, bs), _decay_lambda=lambda: lam,
                                     _span_log_decay=mg.DeltaMinGRU._span_log_decay,
                                     _warned_fp32_decay_saturation=True)
        y, HT = mg.DeltaMinGRU._forward_chunked_gated(shim, Q.new_empty(Bq, Tq, 1), H0, dtt)
        return y.permute(0, 2, 1, 3), HT

    for name, (B, H, T, nh, dk, dv, chunk, big) in {
        "deltagated_small": (2, 2, 11, 1, 8, 8, 4, False),
        "deltagated_nh2": (1, 2, 13, 2, 4, 4, 5, False),
        "deltagated_c16": (1, 2, 40, 1, 16, 16, 16, False),
        "deltagated_saturated": (1, 2, 30, 1, 8, 8, 8, True),
    }.items():
        if only is not None and name not in only:
            continue
        g = torch.Generator().manual_seed(41)
        Q = torch.randn(B, H, T, dk, generator=g, dtype=dt).requires_grad_(True)
        K = F.normalize(torch.randn(B, H, T, nh, dk, generator=g, dtype=dt), dim=-1).requires_grad_(True)
        V = torch.randn(B, H, T, nh, dv, generator=g, dtype=dt).requires_grad_(True)
        beta = (2 * torch.sigmoid(torch.randn(B, H, T, nh, generator=g, dtype=dt))).requires_grad_(True)
        H0 = (torch.randn(B, H, dk, dv, generator=g, dtype=dt) * 0.1).requires_grad_(True)
        lam = (torch.rand(H, generator=g, dtype=dt) + 0.1).requires_grad_(True)
        dtt = torch.rand(B, T, generator=g, dtype=dt) * 2
        if big:  # a few gaps large enough to wipe the memory
            dtt[:, 7] = 1e4
            dtt[:, 19] = 80.0
        dtt.requires_grad_(True)
        y, HT = delta_gated_ref(Q, K, V, beta, H0, lam, dtt, chunk)
        (gy, gHT), gs = grads([y, HT], [Q, K, V, beta, H0, lam, dtt], 1234)
        dQ, dK, dV, dbeta, dH0, dlam, ddt = gs
        save(name, Q=Q, K=K, V=V, beta=beta, H0=H0, lam=lam, dt=dtt, y=y, H_T=HT, grad_y=gy,
             grad_H_T=gHT, dQ=dQ, dK=dK, dV=dV, dbeta=dbeta, dH0=dH0, dlam=dlam, ddt=ddt,
             chunk=torch.tensor(chunk))

    # ------------------------------------------------------------ modules
    import json

    module_cases = {
        "module_mingru": ("MinGRU", dict(input_size=8, hidden_size=16, learnable_h0=True), False),
        "module_mingru_decay": ("MinGRU", dict(input_size=8, hidden_size=16, decay="learnable",
                                                decay_rate=0.5), True),
        "module_signed": ("SignedMinGRU", dict(input_size=8, hidden_size=16, coupled=True,
                                                learnable_h0=True, decay="fixed"), True),
        "module_rotation": ("RotationMinGRU", dict(input_size=8, hidden_size=16, decay="fixed"), True),
        "module_rotation_nosnap": ("RotationMinGRU", dict(input_size=8, hidden_size=12, snap=None), False),
        "module_givens": ("GivensMinGRU", dict(input_size=8, hidden_size=32, block_size=8, rounds=3,
                                               decay="learnable"), True),
        "module_givens_k4": ("GivensMinGRU", dict(input_size=8, hidden_size=16, block_size=4,
                                                  rounds=2), False),
        "module_delta": ("DeltaMinGRU", dict(input_size=8, hidden_size=32, n_heads=2, chunk_size=8), False),
        "module_stack_mixed": ("MinGRUStack", dict(input_size=6, d_model=16, n_layers=3,
                                                   mixer=["log", "signed", "givens"],
                                                   mixer_kwargs={"givens": {"block_size": 4,
                                                                            "rounds": 2}}), False),
        "module_stack_delta": ("MinGRUStack", dict(input_size=8, d_model=16, n_layers=2,
                                                   mixer=["delta", "rotation"],
                                                   mixer_kwargs={"delta": {"n_heads": 2,
                                                                           "chunk_size": 16}}), False),
        # two micro-steps per token at the default chunk_size=64 (nh * chunk = 128)
        "module_delta_nh2": ("DeltaMinGRU", dict(input_size=8, hidden_size=32, n_heads=2, nh=2), False),
        # d_k = d_v = 128 per head (hidden 256 over 2 heads; d_model=512 over 4 heads
        # runs the same kernels per head)
        "module_delta_d128": ("DeltaMinGRU", dict(input_size=16, hidden_size=256, n_heads=2), False),
        # decay active: the reference's eager _forward_chunked_gated
        "module_delta_decay": ("DeltaMinGRU", dict(input_size=8, hidden_size=32, n_heads=2,
                                                   chunk_size=16, decay="learnable"), True),
        "module_delta_decay_fixed": ("DeltaMinGRU", dict(input_size=8, hidden_size=16, n_heads=2,
                                                         nh=2, decay="fixed", decay_rate=0.3), True),
    }
    long_t = {"module_delta_nh2": 150, "module_delta_d128": 70,  # several chunks
              "module_delta_decay": 50, "module_delta_decay_fixed": 40}
    for name, (cls_name, kwargs, use_dt) in module_cases.items():
        if only is not None and name not in only:
            continue
        torch.manual_seed(101)
        mod = getattr(mg, cls_name)(**kwargs).double()
        B, T = 3, long_t.get(name, 37)
        g = torch.Generator().manual_seed(102)
        x = torch.randn(B, T, kwargs["input_size"], generator=g, dtype=dt).requires_grad_(True)
        dtv = (torch.rand(B, T, generator=g, dtype=dt) * 2) if use_dt else None
        if cls_name == "MinGRUStack":
            out, _ = mod(x)
        elif cls_name == "DeltaMinGRU":
            out = mod(x) if dtv is None else mod(x, None, dtv)
        else:
            out = mod(x, None, dtv)
        cot = torch.randn(out.shape, generator=torch.Generator().manual_seed(1234), dtype=dt)
        params = list(mod.named_parameters())
        grads = torch.autograd.grad((out * cot).sum(), [x] + [p for _, p in params],
                                    allow_unused=True)
        arrays = {"x": x, "out": out, "cot": cot, "dx": grads[0]}
        if dtv is not None:
            arrays["delta_t"] = dtv
        for (pn, pv), gp in zip(params, grads[1:]):
            arrays["grad." + pn] = torch.zeros_like(pv) if gp is None else gp
        for k, v in mod.state_dict().items():
            arrays["sd." + k] = v
        np.savez_compressed(HERE / f"{name}.npz",
                            meta=np.array(json.dumps({"cls": cls_name, "kwargs": kwargs})),
                            **{k: _np(v) for k, v in arrays.items()})

    # -------------------------------------------------------------- steps
    # Each mixer's step() over a few tokens (the streaming path), from a
    # seeded module; with decay the time gaps are passed per token.
    step_cases = {
        "step_mingru": ("MinGRU", dict(input_size=6, hidden_size=16, learnable_h0=True), False),
        "step_mingru_decay": ("MinGRU", dict(input_size=6, hidden_size=16, decay="learnable"), True),
        "step_signed": ("SignedMinGRU", dict(input_size=6, hidden_size=16, coupled=True,
                                             learnable_h0=True), False),
        "step_signed_decay": ("SignedMinGRU", dict(input_size=6, hidden_size=16,
                                                   decay="fixed"), True),
        "step_rotation": ("RotationMinGRU", dict(input_size=6, hidden_size=16, snap=None), False),
        "step_rotation_decay": ("RotationMinGRU", dict(input_size=6, hidden_size=12,
                                                       decay="learnable"), True),
        "step_givens": ("GivensMinGRU", dict(input_size=6, hidden_size=32, block_size=8,
                                             rounds=3), False),
        "step_givens_decay": ("GivensMinGRU", dict(input_size=6, hidden_size=16, block_size=4,
                                                   rounds=2, decay="fixed"), True),
        "step_delta": ("DeltaMinGRU", dict(input_size=6, hidden_size=16, n_heads=2, nh=2), False),
        "step_delta_decay": ("DeltaMinGRU", dict(input_size=6, hidden_size=16, n_heads=2,
                                                 decay="learnable"), True),
    }
    for name, (cls_name, kwargs, use_dt) in step_cases.items():
        if only is not None and name not in only:
            continue
        torch.manual_seed(201)
        mod = getattr(mg, cls_name)(**kwargs).double()
        B, T = 3, 6
        g = torch.Generator().manual_seed(202)
        xs = torch.randn(B, T, kwargs["input_size"], generator=g, dtype=dt)
        dts = torch.rand(B, T, generator=g, dtype=dt) * 2 if use_dt else None
        h, ys, hs = None, [], []
        with torch.no_grad():
            for t in range(T):
                r = mod.step(xs[:, t], h, None if dts is None else dts[:, t])
                if cls_name == "DeltaMinGRU":
                    y, h = r
                else:
                    y = h = r
                ys.append(y)
                hs.append(h)
        arrays = {"x": xs, "y": torch.stack(ys, 1), "h": torch.stack(hs, 1)}
        if dts is not None:
            arrays["delta_t"] = dts
        for k2, v in mod.state_dict().items():
            arrays["sd." + k2] = v
        np.savez_compressed(HERE / f"{name}.npz",
                            meta=np.array(json.dumps({"cls": cls_name, "kwargs": kwargs})),
                            **{k2: _np(v) for k2, v in arrays.items()})

    if only is None or "module_delta_ref_fixture" in only:
        ref_fixture(Path(args.ref).parent / "tests" / "fixtures" / "delta_mingru_decay_none_golden.json")
    print(f"wrote fixtures to {HERE}")


def ref_fixture(src: Path) -> None:
    """The reference's own DeltaMinGRU golden (tests/fixtures/
    delta_mingru_decay_none_golden.json, checked by tests/test_mixers.py:403-437:
    DeltaMinGRU(8, 6, n_heads=2, nh=2) from seed 42, its state_dict, input,
    output and the gradients of output.sum()) in this directory's module-fixture
    layout, so the module tests gate against it too."""
    import json

    f = json.loads(src.read_text())
    arrays = {"x": np.array(f["x"], np.float32), "out": np.array(f["output"], np.float32),
              "dx": np.array(f["x_grad"], np.float32)}
    arrays["cot"] = np.ones_like(arrays["out"])
    for k in f["state_dict_keys"]:
        arrays["sd." + k] = np.array(f["state_dict"][k], np.float32)
    for k, v in f["param_grads"].items():
        arrays["grad." + k] = np.array(v, np.float32)
    meta = {"cls": "DeltaMinGRU", "kwargs": {"input_size": f["D_IN"], "hidden_size": f["D_H"],
                                             "n_heads": f["n_heads"], "nh": f["nh"]},
            "seed": f["seed"], "dtype": "float32",
            "source": "reference tests/fixtures/delta_mingru_decay_none_golden.json"}
    np.savez_compressed(HERE / "module_delta_ref_fixture.npz", meta=np.array(json.dumps(meta)),
                        **arrays)


def eager_dev(ref: str) -> None:
    import json

    os.environ["MINGRU_SCAN"] = "eager"
    sys.path.insert(0, ref)
    sys.path.insert(0, str(HERE.parent))
    import torch
    from mingru import min_gru as mg

    import cases as C

    torch.set_num_threads(os.cpu_count() or 1)

    def t(x, dtype, grad=False):
        r = torch.as_tensor(np.asarray(x), dtype=dtype)
        return r.requires_grad_(True) if grad else r

    # ---- delta: DeltaMinGRU._forward_chunked through the raw-tensor shim
    def delta_eager(d, chunk, dtype):
        Q, K, V, beta = (t(d[k], dtype, True) for k in ("Q", "K", "V", "beta"))
        H0 = t(d["H0"], dtype, True)
        Bq, nH, Tq, dk = Q.shape
        nh, dv = K.shape[3], V.shape[4]
        q = Q.permute(0, 2, 1, 3)
        ks = list(K.permute(0, 2, 3, 1, 4).unbind(2))
        vs = list(V.permute(0, 2, 3, 1, 4).unbind(2))
        bs = list(beta.permute(0, 2, 3, 1).unbind(2))
        shim = types.SimpleNamespace(nh=nh, n_heads=nH, d_k=dk, d_v=dv, chunk_size=chunk,
                                     _coeffs=lambda x: (q, ks, vs, bs))
        y, HT = mg.DeltaMinGRU._forward_chunked(shim, Q.new_empty(Bq, Tq, 1), H0)
        y = y.permute(0, 2, 1, 3)
        gs = torch.autograd.grad((y * t(d["grad_y"], dtype)).sum() + (HT * t(d["grad_H_T"], dtype)).sum(),
                                 [Q, K, V, beta, H0])
        out = {"y": y, "H_T": HT}
        out.update(zip(C.DELTA_NAMES, gs))
        return {k: v.detach().double().numpy() for k, v in out.items()}

    def dev_of(f32, f64):
        return {k: float(np.max(np.abs(f32[k] - f64[k]))) if f64[k].size else 0.0 for k in f64}

    res: dict[str, dict[str, float]] = {}

    def delta_case(key, d, chunk):
        res[key] = dev_of(delta_eager(d, chunk, torch.float32), delta_eager(d, chunk, torch.float64))
        print(key, {k: f"{v:.2e}" for k, v in res[key].items()}, flush=True)

    for case in C.DELTA_CASES:
        delta_case(C.case_key("delta_fp32", case), C.delta_case_inputs("fp32", case), case[-1])
    for case in C.DELTA_TC_CASES:
        delta_case(C.case_key("delta_bf16", case), C.delta_case_inputs("bf16", case), case[-1])
    def delta_gated_eager(d, lam, dtt, chunk, dtype):
        Q, K, V, beta, H0 = (t(d[k], dtype, True) for k in ("Q", "K", "V", "beta", "H0"))
        lm, dd = t(lam, dtype, True), t(dtt, dtype, True)
        Bq, nH, Tq, dk = Q.shape
        nh, dv = K.shape[3], V.shape[4]
        q = Q.permute(0, 2, 1, 3)
        ks = list(K.permute(0, 2, 3, 1, 4).unbind(2))
        vs = list(V.permute(0, 2, 3, 1, 4).unbind(2))
        bs = list(beta.permute(0, 2, 3, 1).unbind(2))
        shim = types.SimpleNamespace(nh=nh, n_heads=nH, d_k=dk, d_v=dv, chunk_size=chunk,
                                     _coeffs=lambda x: (q, ks, vs, bs), _decay_lambda=lambda: lm,
                                     _span_log_decay=mg.DeltaMinGRU._span_log_decay,
                                     _warned_fp32_decay_saturation=True)
        y, HT = mg.DeltaMinGRU._forward_chunked_gated(shim, Q.new_empty(Bq, Tq, 1), H0, dd)
        y = y.permute(0, 2, 1, 3)
        gs = torch.autograd.grad((y * t(d["grad_y"], dtype)).sum() + (HT * t(d["grad_H_T"], dtype)).sum(),
                                 [Q, K, V, beta, H0, lm, dd])
        out = {"y": y, "H_T": HT}
        out.update(zip(C.DELTA_NAMES + ["dlam", "ddt"], gs))
        return {k: v.detach().double().numpy() for k, v in out.items()}

    for case in C.DELTA_GATED_CASES:
        d, lam, dtt = C.delta_gated_inputs(case, seed=sum(case))
        key = C.case_key("delta_gated", case)
        res[key] = dev_of(delta_gated_eager(d, lam, dtt, case[-1], torch.float32),
                          delta_gated_eager(d, lam, dtt, case[-1], torch.float64))
        print(key, {k: f"{v:.2e}" for k, v in res[key].items()}, flush=True)
    delta_case("delta_full_fp32", C.delta_full_inputs(False), C.DELTA_FULL[-1])
    delta_case("delta_full_bf16", C.delta_full_inputs(True), C.DELTA_FULL[-1])
    for f in sorted(HERE.glob("delta_*.npz")):
        with np.load(f) as z:
            g = {k: z[k] for k in z.files}
        e32 = delta_eager(g, int(g["chunk"]), torch.float32)
        res["golden:" + f.stem] = {k: float(np.max(np.abs(e32[k] - g[k]))) for k in e32}

    # ---- angle: per-step matrices from the plane angles, matrix_affine_scan
    def angle_eager(d, hs, hd, dtype):
        th, sc, ga, bb, h0 = (t(d[k], dtype, True) for k in ("theta", "scale", "gamma", "b", "h0"))
        perm, sgn, p2p = (torch.as_tensor(np.asarray(d[k])) for k in ("perm", "sgn", "p2p"))
        B, T, n, R, half = th.shape
        k = bb.shape[-1]
        eye = torch.eye(k, dtype=dtype)
        M = eye.expand(B, T, n, k, k)
        if hs and k == 2:
            S = torch.stack([torch.stack([torch.ones_like(sc), torch.zeros_like(sc)], -1),
                             torch.stack([torch.zeros_like(sc), sc], -1)], -2)
            M = S
        for r in range(R):
            ang = th[:, :, :, r, :][..., p2p[r].long()]  # (B, T, n, k): angle of row p's plane
            P = torch.nn.functional.one_hot(perm[r].long(), k).to(dtype)  # P[p, perm[p]] = 1
            # row p of the round: cos(a_p) e_p + sgn_p sin(a_p) e_perm(p)
            Rm = torch.diag_embed(torch.cos(ang)) + (sgn[r].to(dtype) * torch.sin(ang))[..., None] * P
            M = Rm @ M
        if hd:
            M = ga[..., None, None] * M
        Ab, Bb = mg.matrix_affine_scan(M, bb.unsqueeze(-1))
        h = torch.einsum("btnij,bnj->btni", Ab, h0) + Bb.squeeze(-1)
        gs = torch.autograd.grad((h * t(d["grad_h"], dtype)).sum(), [th, sc, ga, bb, h0],
                                 allow_unused=True)
        out = {"h": h}
        for name, gg, x in zip(["dtheta", "dscale", "dgamma", "db", "dh0"], gs, [th, sc, ga, bb, h0]):
            out[name] = torch.zeros_like(x) if gg is None else gg
        return {k2: v.detach().double().numpy() for k2, v in out.items()}

    def angle_case(key, d, hs, hd):
        res[key] = dev_of(angle_eager(d, hs, hd, torch.float32), angle_eager(d, hs, hd, torch.float64))
        print(key, {k: f"{v:.2e}" for k, v in res[key].items()}, flush=True)

    for case in C.ANGLE_CASES:
        angle_case(C.case_key("angle", case), C.angle_case_inputs(case), case[5], case[6])
    # config 4: the deviation of the first batch row stands for all eight
    # (the rows are i.i.d.; eager fp64 of all eight would need ~80 GB of host memory)
    angle_case("angle_full_config4", C.angle_full_config4(rows=1), 0, 1)
    for f in sorted(list(HERE.glob("givens_*.npz")) + list(HERE.glob("rotation*.npz"))):
        with np.load(f) as z:
            g = {k: z[k] for k in z.files}
        hs, hd = (int(x) for x in g["flags"])
        e32 = angle_eager(g, hs, hd, torch.float32)
        ref = {"h": g["h"], "dtheta": g["dtheta"], "dgamma": g["dgamma"], "db": g["db"],
               "dh0": g["dh0"], "dscale": g.get("dscale", np.zeros_like(e32["dscale"]))}
        res["golden:" + f.stem] = {k: float(np.max(np.abs(e32[k] - ref[k]))) for k in ref}

    out = HERE / "eager_dev.json"
    out.write_text(json.dumps(res, indent=1, sort_keys=True) + "\n")
    print(f"wrote {out} ({len(res)} cases)")


if __name__ == "__main__":
    main()
