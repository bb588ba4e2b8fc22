"""Seeded inputs shared by the GPU parity tests and the fixture generator.

Both the tests (on the GPU box) and ``tests/golden/make_golden.py`` (here,
with the reference importable) build their inputs with these functions, so
the eager fp32-vs-fp64 deviations the generator records in
``tests/golden/eager_dev.json`` belong to exactly the inputs the tests run.
numpy's PCG64 stream is the same on every platform."""

from __future__ import annotations

import math

import numpy as np


def _f32(x):
    return np.asarray(x).astype(np.float32).astype(np.float64)


def _bf16(x):
    """Round to bfloat16 (round to nearest even), returned as float64."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


# ------------------------------------------------------------------ delta --

DELTA_NAMES = ["dQ", "dK", "dV", "dbeta", "dH0"]

# (B, H, T, nh, dk, dv, chunk): fp32 inputs against the fp64 oracle
DELTA_CASES = [
    (1, 2, 100, 1, 64, 64, 64), (2, 1, 77, 2, 32, 32, 32), (1, 2, 130, 1, 16, 16, 16),
    (2, 2, 19, 1, 8, 8, 8), (1, 1, 65, 1, 64, 32, 64), (1, 3, 40, 4, 8, 16, 16),
    (1, 1, 1, 1, 4, 4, 4),
    # wider than the 64-micro-step tiles: nh * chunk = 128 (the kernels run
    # shorter chunks), d_k = d_v = 128 (d_v in two column blocks), an odd chunk
    (1, 2, 150, 2, 16, 16, 64), (1, 2, 100, 2, 64, 64, 64), (1, 1, 70, 1, 128, 128, 64),
    (1, 1, 30, 3, 8, 8, 50),
]
# bf16 inputs on the tensor-core kernels: value-column splits of 2 (d_v > 32,
# few heads) and 1 (many heads, or d_v <= 32), padded d_k / d_v / chunk rows,
# nh > 1, ragged T.
DELTA_TC_CASES = [
    (1, 2, 100, 1, 64, 64, 64), (2, 1, 77, 2, 32, 32, 32), (1, 2, 130, 1, 16, 16, 16),
    (2, 2, 19, 1, 8, 8, 8), (1, 1, 65, 1, 64, 32, 64), (1, 3, 40, 4, 8, 16, 16),
    (1, 2, 90, 1, 48, 40, 64), (10, 8, 70, 1, 64, 64, 64), (1, 1, 1, 1, 8, 8, 64),
    # nh * chunk = 128 (tensor cores with 32-token chunks) and d_k = d_v = 128
    # (CUDA-core kernels on bf16 inputs, d_v in two column blocks)
    (1, 2, 150, 2, 64, 64, 64), (1, 1, 70, 1, 128, 128, 64),
]
# BASELINE config 5 at full size: B=8, H=8, T=8192, d_k=d_v=64, chunk=64
DELTA_FULL = (8, 8, 8192, 1, 64, 64, 64)


def delta_inputs(B, H, T, nh, dk, dv, seed):
    """fp32-representable inputs (float64 arrays) of one delta case."""
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
    return {k: _f32(v) for k, v in d.items()}


def delta_bf16_inputs(case, seed):
    """Inputs of a bf16 case: Q, K, V, beta and grad_y rounded to bf16."""
    B, H, T, nh, dk, dv, chunk = case
    d = delta_inputs(B, H, T, nh, dk, dv, seed)
    for k in ("Q", "K", "V", "beta", "grad_y"):
        d[k] = _bf16(d[k])
    return d


def delta_full_inputs(bf16: bool):
    if bf16:
        d = delta_bf16_inputs(DELTA_FULL, seed=5)
    else:
        d = delta_inputs(*DELTA_FULL[:6], seed=0)
    d["H0"][:] = 0.0
    return d


def delta_case_inputs(kind: str, case):
    """The inputs a delta test runs for `kind` in {"fp32", "bf16"}."""
    if kind == "fp32":
        return delta_inputs(*case[:6], seed=sum(case))
    return delta_bf16_inputs(case, seed=sum(case) + 1)


# decay-active delta: (B, H, T, nh, dk, dv, chunk)
DELTA_GATED_CASES = [
    (2, 2, 100, 1, 32, 32, 32), (1, 2, 150, 2, 16, 16, 64), (1, 1, 70, 1, 64, 64, 64),
    (2, 3, 45, 3, 8, 16, 10), (1, 2, 90, 1, 16, 80, 64),
    # d_k = 96 (the CUDA-core kernels with decay) and one token with nh = 2
    (1, 2, 60, 1, 96, 32, 16), (2, 1, 1, 2, 16, 16, 8),
]


def delta_gated_inputs(case, seed):
    """Inputs of a decay-active case: the delta inputs (beta = 2 sigmoid, as
    DeltaMinGRU builds it), per-head lambda and per-token gaps dt, one gap
    large enough to wipe the memory."""
    B, H, T, nh, dk, dv, chunk = case
    rng = np.random.default_rng(seed)
    K = rng.standard_normal((B, H, T, nh, dk))
    K /= np.linalg.norm(K, axis=-1, keepdims=True)
    d = {
        "Q": rng.standard_normal((B, H, T, dk)),
        "K": K,
        "V": rng.standard_normal((B, H, T, nh, dv)),
        "beta": 2 / (1 + np.exp(-rng.standard_normal((B, H, T, nh)))),
        "H0": rng.standard_normal((B, H, dk, dv)) * 0.1,
        "grad_y": rng.standard_normal((B, H, T, dv)),
        "grad_H_T": rng.standard_normal((B, H, dk, dv)),
    }
    lam = rng.random(H) * 0.5 + 0.05
    dtt = rng.random((B, T)) * 2
    dtt[:, T // 3] = 1e3
    return {k: _f32(v) for k, v in d.items()}, _f32(lam), _f32(dtt)


def case_key(prefix: str, case) -> str:
    return prefix + ":" + ",".join(str(x) for x in case)


# ------------------------------------------------------------------ angle --

# (B, T, n, R, k, has_scale, has_decay, meta)
ANGLE_CASES = [
    (2, 13, 3, 1, 2, 1, 0, "brickwall"), (2, 100, 33, 1, 2, 1, 1, "brickwall"),
    (1, 64, 5, 2, 2, 0, 1, "brickwall"), (2, 37, 40, 3, 4, 0, 1, "brickwall"),
    (1, 50, 9, 4, 4, 0, 0, "brickwall"), (2, 70, 33, 2, 8, 0, 1, "brickwall"),
    (1, 45, 7, 3, 8, 0, 1, "brickwall"), (1, 23, 3, 4, 8, 0, 0, "brickwall"),
    (1, 20, 3, 3, 8, 0, 1, "shuffled"), (1, 15, 2, 2, 16, 0, 1, "brickwall"),
    (1, 9, 2, 5, 4, 0, 1, "brickwall"), (2, 1, 4, 2, 8, 0, 1, "brickwall"),
]


def brickwall(R: int, k: int):
    """(perm, sgn, p2p) of the brick-wall plane layout (round r pairs (i, i+1
    mod k) for i = r%2, r%2+2, ...; sgn -1 on i and +1 on i+1)."""
    perm = np.zeros((R, k), np.int32)
    sgn = np.zeros((R, k), np.float32)
    p2p = np.zeros((R, k), np.int32)
    for r in range(R):
        for m, i in enumerate(range(r % 2, k, 2)):
            i %= k
            j = (i + 1) % k
            perm[r, i], perm[r, j] = j, i
            sgn[r, i], sgn[r, j] = -1.0, 1.0
            p2p[r, i], p2p[r, j] = m, m
    return perm, sgn, p2p


def angle_inputs(B, T, n, R, k, seed, *, has_scale, has_decay, meta="brickwall"):
    rng = np.random.default_rng(seed)
    d = {
        "theta": (rng.random((B, T, n, R, k // 2)) * 2 - 1) * math.pi,
        "scale": np.tanh(rng.standard_normal((B, T, n))) if has_scale else np.ones((B, T, n)),
        "gamma": 1 / (1 + np.exp(-rng.standard_normal((B, T, n)))) if has_decay else np.ones((B, T, n)),
        "b": rng.standard_normal((B, T, n, k)),
        "h0": rng.standard_normal((B, n, k)),
        "grad_h": rng.standard_normal((B, T, n, k)),
    }
    for key in ("theta", "scale", "gamma", "b", "h0", "grad_h"):
        d[key] = _f32(d[key])
    perm, sgn, p2p = brickwall(R, k)
    if meta == "shuffled":  # a valid pairing that is not the brick-wall layout
        for r in range(R):
            order = rng.permutation(k)
            for m in range(k // 2):
                i, j = int(order[2 * m]), int(order[2 * m + 1])
                perm[r, i], perm[r, j] = j, i
                sgn[r, i], sgn[r, j] = -1.0, 1.0
                p2p[r, i], p2p[r, j] = m, m
    d.update(perm=perm, sgn=sgn, p2p=p2p)
    return d


def angle_case_inputs(case):
    B, T, n, R, k, hs, hd, meta = case
    return angle_inputs(B, T, n, R, k, seed=sum(case[:5]), has_scale=hs, has_decay=hd, meta=meta)


def angle_full_config4(rows: int = 8):
    """BASELINE config 4 (first `rows` batch rows of the B=8 inputs): T=4096,
    n=128, k=8, R=2 with the wrap-around plane (7, 0) angle fixed to 0."""
    d = angle_inputs(8, 4096, 128, 2, 8, seed=0, has_scale=0, has_decay=1)
    d["theta"][:, :, :, 1, 3] = 0.0
    d["h0"][:] = 0.0
    if rows < 8:
        for key in ("theta", "scale", "gamma", "b", "h0", "grad_h"):
            d[key] = d[key][:rows]
    return d


# ---------------------------------------------------------------- gates --


def gate(bar: dict, dev: dict | None, name: str) -> dict:
    """Tolerance of one compared tensor: the parity bar, with its absolute part
    raised to 10x the reference eager path's own fp32-vs-fp64 deviation on the
    same inputs where that is larger (the reference parity runner's rule,
    triton_scans.py:3303-3330)."""
    own = 0.0 if dev is None else float(dev.get(name, 0.0))
    return dict(rtol=bar["rtol"], atol=max(bar["atol"], 10.0 * own))


def report(label: str, got, ref, dev: dict | None, name: str) -> str:
    """One line: kernel vs fp64, eager fp32 vs fp64, and their ratio."""
    err = float(np.max(np.abs(np.asarray(got) - np.asarray(ref)))) if np.size(ref) else 0.0
    own = None if dev is None else dev.get(name)
    ratio = "" if not own else f"  kernel/eager32 {err / own:.3g}"
    own_s = "n/a" if own is None else f"{own:.3g}"
    return f"{label} {name}: |kernel-fp64| {err:.3g}  |eager32-fp64| {own_s}{ratio}"
