"""Python front end of the CPU oracle. TEST INFRASTRUCTURE ONLY.

Imported by ``tests/``, ``__graft_entry__.smoke()`` (as the checker) and the
CPU-baseline leg of ``bench.py``; never by the product package
``mingru_b200``. It wraps ``liboracle_scan.so`` (sequential C restatements of
the reference algorithms, see ``scan_oracle.c``) with numpy in / numpy out
functions named after the reference ops. ``dtype`` selects the arithmetic:
``np.float64`` (default, the ground truth GPU results are gated against) or
``np.float32`` (the timed CPU baseline).
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle_scan.so"

_lib = None


def build() -> Path:
    """Compile ``liboracle_scan.so`` with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
    return _lib


def set_threads(n: int) -> int:
    """Use n OpenMP threads in the oracle loops; returns the count in effect."""
    lib().orc_set_threads(ctypes.c_int(int(n)))
    return int(lib().orc_get_threads())


def _suffix(dtype) -> str:
    dt = np.dtype(dtype)
    if dt == np.float64:
        return "f64"
    if dt == np.float32:
        return "f32"
    raise TypeError(f"oracle supports float32/float64, got {dt}")


def _arr(x, dtype) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x), dtype=dtype)


def _p(x: np.ndarray):
    return x.ctypes.data_as(ctypes.c_void_p)


_I = ctypes.c_int64


def parallel_scan_log(log_coeffs, log_values, dtype=np.float64):
    """h (B,T,D) of min_gru.parallel_scan_log as the sequential recurrence."""
    lc, lv = _arr(log_coeffs, dtype), _arr(log_values, dtype)
    B, T, D = lc.shape
    assert lv.shape == (B, T + 1, D)
    h = np.empty_like(lc)
    getattr(lib(), f"orc_log_scan_fwd_{_suffix(dtype)}")(_p(lc), _p(lv), _p(h), _I(B), _I(T), _I(D))
    return h


def parallel_scan_log_bwd(log_coeffs, log_values, grad_h, dtype=np.float64):
    """(dlog_coeffs, dlog_values) for upstream grad ``grad_h``."""
    lc, lv, gh = _arr(log_coeffs, dtype), _arr(log_values, dtype), _arr(grad_h, dtype)
    B, T, D = lc.shape
    dlc, dlv = np.empty_like(lc), np.empty_like(lv)
    getattr(lib(), f"orc_log_scan_bwd_{_suffix(dtype)}")(
        _p(lc), _p(lv), _p(gh), _p(dlc), _p(dlv), _I(B), _I(T), _I(D)
    )
    return dlc, dlv


def _softplus(x):
    return np.maximum(x, 0) + np.log1p(np.exp(-np.abs(x)))


def mingru_gate_logs(k, x, log_h0):
    """(log_coeffs, log_values) MinGRU.forward builds from the gate and
    candidate pre-activations k = linear_z(x), x~ = linear_h(x) and log h_0
    (B, D) (reference min_gru.py:1383-1397, log_g at min_gru.py:751-752):
    log a = -softplus(k), log b = -softplus(-k) + log_g(x~)."""
    k, x, lh0 = (np.asarray(t, dtype=np.float64) for t in (k, x, log_h0))
    log_g = np.where(x >= 0, np.log(np.maximum(x, 0) + 0.5), -_softplus(-x))
    lc = -_softplus(k)
    lv = np.concatenate([lh0[:, None, :], -_softplus(-k) + log_g], axis=1)
    return lc, lv


def mingru_gate_scan(k, x, log_h0):
    """h of parallel_scan_log over MinGRU's gate prologue (fp64)."""
    return parallel_scan_log(*mingru_gate_logs(k, x, log_h0))


def mingru_gate_scan_bwd(k, x, log_h0, grad_h):
    """(dk, dx~, dlog_h0): the log-scan adjoint chained through the prologue
    (d log a/dk = -sigmoid(k), d log b/dk = sigmoid(-k), d log_g/dx~ =
    1/(x~ + 1/2) for x~ >= 0 else sigmoid(-x~))."""
    k, x = np.asarray(k, dtype=np.float64), np.asarray(x, dtype=np.float64)
    lc, lv = mingru_gate_logs(k, x, log_h0)
    dlc, dlv = parallel_scan_log_bwd(lc, lv, grad_h)
    with np.errstate(over="ignore"):
        sk = 1.0 / (1.0 + np.exp(-k))
        fx = np.where(x >= 0, 1.0 / (np.maximum(x, 0) + 0.5), 1.0 / (1.0 + np.exp(x)))
    dk = -sk * dlc + (1.0 - sk) * dlv[:, 1:]
    return dk, fx * dlv[:, 1:], dlv[:, 0]


def linear_scan(a, b, dtype=np.float64):
    """(A, Bc) of min_gru.linear_scan."""
    a, b = _arr(a, dtype), _arr(b, dtype)
    B, T, D = a.shape
    A, Bc = np.empty_like(a), np.empty_like(b)
    getattr(lib(), f"orc_linear_scan_fwd_{_suffix(dtype)}")(
        _p(a), _p(b), _p(A), _p(Bc), _I(B), _I(T), _I(D)
    )
    return A, Bc


def linear_scan_bwd(a, A, Bc, gA, gBc, dtype=np.float64):
    """(da, db) given the forward input ``a`` and outputs ``A``, ``Bc``."""
    a, A, Bc, gA, gBc = (_arr(x, dtype) for x in (a, A, Bc, gA, gBc))
    B, T, D = a.shape
    da, db = np.empty_like(a), np.empty_like(a)
    getattr(lib(), f"orc_linear_scan_bwd_{_suffix(dtype)}")(
        _p(a), _p(A), _p(Bc), _p(gA), _p(gBc), _p(da), _p(db), _I(B), _I(T), _I(D)
    )
    return da, db


def matrix_affine_scan(A, Bm, dtype=np.float64):
    """(Abar, Bbar) of min_gru.matrix_affine_scan; A (B,T,n,k,k), Bm (B,T,n,k,v)."""
    A, Bm = _arr(A, dtype), _arr(Bm, dtype)
    B, T, n, k, _ = A.shape
    v = Bm.shape[-1]
    Ab, Bb = np.empty_like(A), np.empty_like(Bm)
    getattr(lib(), f"orc_affine_scan_fwd_{_suffix(dtype)}")(
        _p(A), _p(Bm), _p(Ab), _p(Bb), _I(B), _I(T), _I(n), ctypes.c_int(k), ctypes.c_int(v)
    )
    return Ab, Bb


def matrix_affine_scan_bwd(A, Abar, Bbar, gAbar, gBbar, dtype=np.float64):
    """(dA, dBm) given forward input ``A`` and outputs ``Abar``, ``Bbar``."""
    A, Abar, Bbar, gA, gB = (_arr(x, dtype) for x in (A, Abar, Bbar, gAbar, gBbar))
    B, T, n, k, _ = A.shape
    v = Bbar.shape[-1]
    dA, dB = np.empty_like(A), np.empty_like(Bbar)
    getattr(lib(), f"orc_affine_scan_bwd_{_suffix(dtype)}")(
        _p(A), _p(Abar), _p(Bbar), _p(gA), _p(gB), _p(dA), _p(dB),
        _I(B), _I(T), _I(n), ctypes.c_int(k), ctypes.c_int(v),
    )
    return dA, dB


def matrix_scan(M, b, dtype=np.float64):
    """(A, Bc) of min_gru.matrix_scan (the k=2, v=1 affine scan)."""
    Ab, Bb = matrix_affine_scan(M, np.asarray(b)[..., None], dtype)
    return Ab, Bb[..., 0]


def matrix_scan_bwd(M, A, Bc, gA, gBc, dtype=np.float64):
    dA, dB = matrix_affine_scan_bwd(
        M, A, np.asarray(Bc)[..., None], gA, np.asarray(gBc)[..., None], dtype
    )
    return dA, dB[..., 0]


def angle_scan(theta, scale, gamma, b, h0, perm, sgn, p2p, *, has_scale, has_decay,
               dtype=np.float64):
    """States h (B,T,n,k) of the angle-fused Givens/rotation recurrence."""
    th, sc, ga, bb, h0 = (_arr(x, dtype) for x in (theta, scale, gamma, b, h0))
    pm = np.ascontiguousarray(np.asarray(perm), dtype=np.int32)
    sg = _arr(sgn, dtype)
    pp = np.ascontiguousarray(np.asarray(p2p), dtype=np.int32)
    B, T, n, R, half = th.shape
    k = bb.shape[-1]
    out = np.empty_like(bb)
    getattr(lib(), f"orc_angle_scan_fwd_{_suffix(dtype)}")(
        _p(th), _p(sc), _p(ga), _p(bb), _p(h0), _p(pm), _p(sg), _p(pp), _p(out),
        _I(B), _I(T), _I(n), ctypes.c_int(R), ctypes.c_int(k),
        ctypes.c_int(int(has_scale)), ctypes.c_int(int(has_decay)),
    )
    return out


def angle_scan_bwd(theta, scale, gamma, h0, out, grad_out, perm, sgn, p2p, *, has_scale,
                   has_decay, dtype=np.float64):
    """(dtheta, dscale, dgamma, db, dh0) of the angle-fused recurrence."""
    th, sc, ga, h0, out, go = (_arr(x, dtype) for x in (theta, scale, gamma, h0, out, grad_out))
    pm = np.ascontiguousarray(np.asarray(perm), dtype=np.int32)
    sg = _arr(sgn, dtype)
    pp = np.ascontiguousarray(np.asarray(p2p), dtype=np.int32)
    B, T, n, R, half = th.shape
    k = out.shape[-1]
    dth, dsc, dga = np.empty_like(th), np.empty_like(sc), np.empty_like(ga)
    db, dh0 = np.empty_like(out), np.empty_like(h0)
    getattr(lib(), f"orc_angle_scan_bwd_{_suffix(dtype)}")(
        _p(th), _p(sc), _p(ga), _p(h0), _p(out), _p(go), _p(pm), _p(sg), _p(pp),
        _p(dth), _p(dsc), _p(dga), _p(db), _p(dh0),
        _I(B), _I(T), _I(n), ctypes.c_int(R), ctypes.c_int(k),
        ctypes.c_int(int(has_scale)), ctypes.c_int(int(has_decay)),
    )
    return dth, dsc, dga, db, dh0
