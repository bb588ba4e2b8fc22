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
    args = ap.parse_args()
    os.environ["MINGRU_SCAN"] = "eager"
    sys.path.insert(0, args.ref)
    import torch
    import torch.nn as nn
    import torch.nn.functional as F
    from mingru import min_gru as mg

    torch.set_default_dtype(torch.float64)
    dt = torch.float64

    def save(name, **arrays):
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
    }
    for name, (cls_name, kwargs, use_dt) in module_cases.items():
        torch.manual_seed(101)
        mod = getattr(mg, cls_name)(**kwargs).double()
        B, T = 3, 37
        g = torch.Generator().manual_seed(102)
        x = torch.randn(B, T, kwargs["input_size"], generator=g, dtype=dt).requires_grad_(True)
        dtv = (torch.rand(B, T, generator=g, dtype=dt) * 2) if use_dt else None
        if cls_name == "MinGRUStack":
            out, _ = mod(x)
        elif cls_name == "DeltaMinGRU":
            out = mod(x)
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

    print(f"wrote {len(list(HERE.glob('*.npz')))} fixtures to {HERE}")


if __name__ == "__main__":
    main()
