"""Numpy oracle for DeltaMinGRU's chunked-WY delta rule. TEST INFRASTRUCTURE ONLY.

Used by ``tests/`` and ``bench.py``'s CPU-baseline leg as the checker; never
imported by ``mingru_b200``. Restates, in float64 numpy:

* ``delta_forward``: the chunked WY form of ``DeltaMinGRU._forward_chunked``
  (reference ``src/mingru/min_gru.py:3152-3255``) at the raw-tensor layout of
  ``delta_scan_impl`` (``src/mingru/triton_scans.py:2403-2447``): per chunk of
  C tokens (M = nh*C micro-steps)
      T  = I + strict_lower(K K^T) * beta[col]
      U  = T^{-1} (V - K H)
      y  = Q H + (Q K^T * beta[col] * read_mask) U,  read_mask = tril(C,C) repeated nh times on cols
      H <- H + K^T (beta * U)
* ``delta_sequential``: the token-by-token micro-step recurrence of
  ``DeltaMinGRU.step`` / ``_micro_step`` (min_gru.py:3107-3150, 3611-3688),
      H <- H + beta k (v - k^T H)^T per micro-step,  y_t = q_t^T H after token t,
  an independent restatement the chunked form must agree with;
* ``delta_backward``: the reverse-chunk adjoint of ``_delta_backward_torch``
  (triton_scans.py:473-605).
Layouts: Q (B,H,T,dk); K (B,H,T,nh,dk); V (B,H,T,nh,dv); beta (B,H,T,nh);
H0 (B,H,dk,dv); y (B,H,T,dv).
"""

from __future__ import annotations

import numpy as np
from scipy.linalg import solve_triangular


def _chunk_mats(Kc, bc, C, nh):
    M = Kc.shape[0]
    strict = np.tril(np.ones((M, M)), -1)
    KK = Kc @ Kc.T
    Tm = np.eye(M) + KK * bc[None, :] * strict
    read = np.repeat(np.tril(np.ones((C, C))), nh, axis=1)
    return KK, strict, Tm, read


def delta_forward(Q, K, V, beta, H0, chunk_size):
    Q, K, V, beta, H0 = (np.asarray(x, dtype=np.float64) for x in (Q, K, V, beta, H0))
    B, Hh, T, dk = Q.shape
    nh, dv = K.shape[3], V.shape[4]
    y = np.zeros((B, Hh, T, dv))
    HT = np.zeros((B, Hh, dk, dv))
    for b in range(B):
        for h in range(Hh):
            S = H0[b, h].copy()
            for s0 in range(0, T, chunk_size):
                e = min(s0 + chunk_size, T)
                C = e - s0
                Kc = K[b, h, s0:e].reshape(C * nh, dk)
                Vc = V[b, h, s0:e].reshape(C * nh, dv)
                bc = beta[b, h, s0:e].reshape(C * nh)
                Qc = Q[b, h, s0:e]
                _, _, Tm, read = _chunk_mats(Kc, bc, C, nh)
                U = solve_triangular(Tm, Vc - Kc @ S, lower=True, unit_diagonal=True)
                y[b, h, s0:e] = Qc @ S + ((Qc @ Kc.T) * bc[None, :] * read) @ U
                S = S + Kc.T @ (bc[:, None] * U)
            HT[b, h] = S
    return y, HT


def delta_sequential(Q, K, V, beta, H0):
    Q, K, V, beta, H0 = (np.asarray(x, dtype=np.float64) for x in (Q, K, V, beta, H0))
    B, Hh, T, dk = Q.shape
    nh, dv = K.shape[3], V.shape[4]
    y = np.zeros((B, Hh, T, dv))
    S = H0.copy()
    for t in range(T):
        for j in range(nh):
            k = K[:, :, t, j]  # (B,H,dk)
            v = V[:, :, t, j]
            bt = beta[:, :, t, j][..., None, None]
            kH = np.einsum("bhk,bhkv->bhv", k, S)
            S = S + bt * np.einsum("bhk,bhv->bhkv", k, v - kH)
        y[:, :, t] = np.einsum("bhk,bhkv->bhv", Q[:, :, t], S)
    return y, S


def delta_backward(Q, K, V, beta, H0, dy, dHT, chunk_size):
    """Grads (dQ, dK, dV, dbeta, dH0) of sum(y*dy) + sum(H_T*dHT)."""
    Q, K, V, beta, H0, dy, dHT = (
        np.asarray(x, dtype=np.float64) for x in (Q, K, V, beta, H0, dy, dHT)
    )
    B, Hh, T, dk = Q.shape
    nh, dv = K.shape[3], V.shape[4]
    dQ, dK, dV, dbeta = (np.zeros_like(x) for x in (Q, K, V, beta))
    dH0 = np.zeros_like(H0)
    starts = list(range(0, T, chunk_size))
    for b in range(B):
        for h in range(Hh):
            # forward pass to record chunk-start states
            bounds, S = [], H0[b, h].copy()
            for s0 in starts:
                e = min(s0 + chunk_size, T)
                C = e - s0
                Kc = K[b, h, s0:e].reshape(C * nh, dk)
                Vc = V[b, h, s0:e].reshape(C * nh, dv)
                bc = beta[b, h, s0:e].reshape(C * nh)
                _, _, Tm, _ = _chunk_mats(Kc, bc, C, nh)
                bounds.append(S.copy())
                U = solve_triangular(Tm, Vc - Kc @ S, lower=True, unit_diagonal=True)
                S = S + Kc.T @ (bc[:, None] * U)
            dH = dHT[b, h].copy()
            for ci in range(len(starts) - 1, -1, -1):
                s0 = starts[ci]
                e = min(s0 + chunk_size, T)
                C = e - s0
                Kc = K[b, h, s0:e].reshape(C * nh, dk)
                Vc = V[b, h, s0:e].reshape(C * nh, dv)
                bc = beta[b, h, s0:e].reshape(C * nh)
                Qc = Q[b, h, s0:e]
                Hc = bounds[ci]
                dyc = dy[b, h, s0:e]
                KK, strict, Tm, read = _chunk_mats(Kc, bc, C, nh)
                U = solve_triangular(Tm, Vc - Kc @ Hc, lower=True, unit_diagonal=True)
                Sm = Qc @ Kc.T
                P = Sm * bc[None, :] * read
                dQc = dyc @ Hc.T
                dHc = Qc.T @ dyc
                dP = dyc @ U.T
                dU = P.T @ dyc
                dKl = (bc[:, None] * U) @ dH.T
                dbU = Kc @ dH
                dU = dU + bc[:, None] * dbU
                dbl = (U * dbU).sum(-1)
                dHc = dHc + dH
                dS = dP * bc[None, :] * read
                dbl = dbl + (dP * Sm * read).sum(0)
                dQc = dQc + dS @ Kc
                dKl = dKl + dS.T @ Qc
                G = solve_triangular(Tm.T, dU, lower=False, unit_diagonal=True)
                dT = -(G @ U.T)
                dKl = dKl - G @ Hc.T
                dHc = dHc - Kc.T @ G
                dKK = dT * bc[None, :] * strict
                dbl = dbl + (dT * KK * strict).sum(0)
                dKl = dKl + dKK @ Kc + dKK.T @ Kc
                dQ[b, h, s0:e] = dQc
                dK[b, h, s0:e] = dKl.reshape(C, nh, dk)
                dV[b, h, s0:e] = G.reshape(C, nh, dv)
                dbeta[b, h, s0:e] = dbl.reshape(C, nh)
                dH = dHc
            dH0[b, h] = dH
    return dQ, dK, dV, dbeta, dH0


def gated_sequential_torch(Q, K, V, beta, H0, log_gamma, grad_y=None, grad_HT=None):
    """The decay-active delta rule as its sequential recurrence, in float64
    torch on the CPU, with autograd for the gradients. TEST INFRASTRUCTURE.

    Per token t (``DeltaMinGRU.step`` with decay, reference min_gru.py:
    3611-3688): the incoming state decays once, H <- exp(log_gamma_t) H, then
    the token's nh micro-steps H <- H + beta k (v - k^T H)^T run undecayed,
    and y_t = q_t^T H. ``_forward_chunked_gated`` (min_gru.py:3290-3448) is the
    chunked form of exactly this recurrence. Inputs as ``delta_forward`` plus
    ``log_gamma`` (B, H, T). Returns (y, H_T) and, when ``grad_y`` is given,
    the gradients (dQ, dK, dV, dbeta, dH0, dlog_gamma) of
    sum(y * grad_y) + sum(H_T * grad_HT)."""
    import torch

    ts = [torch.as_tensor(np.asarray(x), dtype=torch.float64).requires_grad_(grad_y is not None)
          for x in (Q, K, V, beta, H0, log_gamma)]
    q, k, v, b, H, lg = ts
    Bn, nH, T, dk = q.shape
    nh = k.shape[3]
    ys = []
    for t in range(T):
        H = torch.exp(lg[:, :, t])[..., None, None] * H
        for m in range(nh):
            km, vm = k[:, :, t, m], v[:, :, t, m]
            kH = torch.einsum("bhk,bhkv->bhv", km, H)
            H = H + b[:, :, t, m][..., None, None] * torch.einsum("bhk,bhv->bhkv", km, vm - kH)
        ys.append(torch.einsum("bhk,bhkv->bhv", q[:, :, t], H))
    y = torch.stack(ys, 2) if ys else q.new_zeros(Bn, nH, 0, v.shape[-1])
    if grad_y is None:
        return y.detach().numpy(), H.detach().numpy()
    gy = torch.as_tensor(np.asarray(grad_y), dtype=torch.float64)
    gH = torch.as_tensor(np.asarray(grad_HT), dtype=torch.float64)
    grads = torch.autograd.grad((y * gy).sum() + (H * gH).sum(), ts, allow_unused=True)
    grads = [torch.zeros_like(x) if g is None else g for x, g in zip(ts, grads)]
    return y.detach().numpy(), H.detach().numpy(), [g.numpy() for g in grads]
