"""Fused per-token recurrence updates behind the mixers' ``step()``.

Each function takes one token's pre-activations (the outputs of the mixer's
linear projections) and the previous state and returns the next state (and,
for the delta rule, the readout) from one kernel of ``libmingru_scan.so``,
where the reference runs a chain of small torch ops per step
(``MinGRU.step`` ... ``DeltaMinGRU.step``, reference ``src/mingru/
min_gru.py:1399-1448, 1858-1901, 2316-2359, 2776-2818, 3611-3688``). No
autograd: ``step()`` is an inference path (``torch.no_grad`` in the
reference too). The arithmetic is fp32 whatever the storage dtype.
"""

from __future__ import annotations

import torch

from . import _lib
from .scan_ops import _dtype_code, _require_cuda

__all__ = ["mingru_step", "signed_step", "rotation_step", "givens_step", "delta_step"]


def _prep(op, *ts, like):
    """CUDA, one dtype, contiguous (None passes through)."""
    present = [t for t in ts if t is not None]
    _require_cuda(op, *present)
    if any(t.dtype != like.dtype for t in present):
        raise ValueError(f"{op}: all inputs must share the dtype {like.dtype}")
    return [None if t is None else t.contiguous() for t in ts]


def _p(t):
    return None if t is None else t.data_ptr()


def _run(op, fn, dev, *args):
    with torch.cuda.device(dev):
        st = fn(*args, torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(st, op)


def mingru_step(k, xh, h_prev, gamma=None):
    """``h = gamma (1 - sigmoid(k)) h_prev + sigmoid(k) g(xh)`` (all ``(B, D)``)."""
    op = "mingru_step"
    k, xh, h_prev, gamma = _prep(op, k, xh, h_prev, gamma, like=k)
    h = torch.empty_like(h_prev)
    B, D = h.shape
    _run(op, _lib.load().mgs_mingru_step, k.device, _p(k), _p(xh), _p(h_prev), _p(gamma), _p(h),
         B, D, _dtype_code(op, k))
    return h


def signed_step(z, s, xh, h_prev, gamma=None, coupled=False):
    """``h = a h_prev + sigmoid(z) xh`` with ``a = gamma tanh(s)``, times
    ``1 - sigmoid(z)`` when coupled (all ``(B, D)``)."""
    op = "signed_step"
    z, s, xh, h_prev, gamma = _prep(op, z, s, xh, h_prev, gamma, like=z)
    h = torch.empty_like(h_prev)
    B, D = h.shape
    _run(op, _lib.load().mgs_signed_step, z.device, _p(z), _p(s), _p(xh), _p(h_prev), _p(gamma),
         int(bool(coupled)), _p(h), B, D, _dtype_code(op, z))
    return h


def rotation_step(theta, u, z, xh, h_prev, gamma=None):
    """Per 2-block: ``h = gamma R(theta) diag(1, tanh u) h_prev + sigmoid(z) xh``;
    ``theta``, ``u``, ``gamma`` ``(B, n)``; ``z``, ``xh``, ``h_prev`` ``(B, 2n)``."""
    op = "rotation_step"
    theta, u, z, xh, h_prev, gamma = _prep(op, theta, u, z, xh, h_prev, gamma, like=theta)
    h = torch.empty_like(h_prev)
    B, n = theta.shape
    _run(op, _lib.load().mgs_rotation_step, theta.device, _p(theta), _p(u), _p(z), _p(xh),
         _p(h_prev), _p(gamma), _p(h), B, n, _dtype_code(op, theta))
    return h


def givens_step(theta, z, xh, h_prev, gamma=None):
    """Per k-block: R brick-wall rounds of plane rotations, ``* gamma``, ``+
    sigmoid(z) xh``; ``theta`` ``(B, n, R, k/2)``, ``gamma`` ``(B, n)``,
    ``z``, ``xh``, ``h_prev`` ``(B, n k)``; k in {2, 4, ..., 64} (powers of 2)."""
    op = "givens_step"
    theta, z, xh, h_prev, gamma = _prep(op, theta, z, xh, h_prev, gamma, like=theta)
    h = torch.empty_like(h_prev)
    B, n, R, half = theta.shape
    _run(op, _lib.load().mgs_givens_step, theta.device, _p(theta), _p(z), _p(xh), _p(h_prev),
         _p(gamma), _p(h), B, n, R, 2 * half, _dtype_code(op, theta))
    return h


def delta_step(q, k, v, beta, H_prev, gamma=None):
    """One token of the delta rule per head: ``H <- gamma H``, then for each of
    the nh micro-steps ``H <- H + beta k (v - k^T H)^T``; readout ``y = H^T q``.
    ``q`` ``(B, H, dk)``, ``k`` ``(B, H, nh, dk)``, ``v`` ``(B, H, nh, dv)``,
    ``beta`` ``(B, H, nh)``, ``gamma`` ``(B, H)``, ``H_prev`` ``(B, H, dk, dv)``.
    Returns ``(y (B, H, dv), H)``."""
    op = "delta_step"
    q, k, v, beta, H_prev, gamma = _prep(op, q, k, v, beta, H_prev, gamma, like=q)
    B, nH, dk = q.shape
    nh, dv = k.shape[2], v.shape[3]
    H = torch.empty_like(H_prev)
    y = torch.empty(B, nH, dv, dtype=q.dtype, device=q.device)
    _run(op, _lib.load().mgs_delta_step, q.device, _p(q), _p(k), _p(v), _p(beta), _p(gamma),
         _p(H_prev), _p(y), _p(H), B, nH, nh, dk, dv, _dtype_code(op, q))
    return y, H
