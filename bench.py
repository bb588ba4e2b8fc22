"""Benchmark of the mingru scan hot path on B200: one JSON line per run.

A "step" is one forward + backward pass of a scan op over one batch of
synthetic inputs of a BASELINE configuration (seeded; the reference publishes
no dataset for this path). Default workload: configuration 2 of the baseline,
``linear_scan`` fwd+bwd at B=16, T=4096, D=1024 in fp32 (the SignedMinGRU
scan). Metric: scan fwd+bwd Gelem/s, elem = one (b, t, d) element.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME]
  python bench.py --impl reference ...   # the reference algorithm on host cores

Multi-GPU runs (torchrun, one rank per GPU) shard by batch: every rank scans
its own batch rows with no collective on the data path (weak scaling: the
per-GPU batch is fixed); the timed region is bracketed by barriers and the
reported time is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
L2_BYTES = 126 * 1024 * 1024
L2_FLUSH_THRESHOLD = 2 * L2_BYTES   # per-step footprint below this is timed with L2 flushes
FLUSH_BYTES = 256 * 1024 * 1024


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


def load_traffic() -> dict[str, float]:
    """DRAM bytes per element per kernel from ncu captures (profiles/traffic.txt)."""
    out: dict[str, float] = {}
    f = ROOT / "profiles" / "traffic.txt"
    if f.exists():
        for line in f.read_text().splitlines():
            parts = line.split("#")[0].split()
            if len(parts) == 2:
                out[parts[0]] = float(parts[1])
    return out


# ------------------------------------------------------------ workloads --


class ScanWorkload:
    """One BASELINE configuration: seeded inputs, one fwd+bwd step through the
    public op + autograd, the algorithmic bytes of each kernel, and the
    CPU-oracle step used for the CPU baseline."""

    name = "?"
    metric_elems_doc = "B*T*D"
    kernels = {"fwd": "?", "bwd": "?"}
    launches_per_step = 2  # one forward kernel + one backward kernel
    compute_dtype = "f32"  # arithmetic of the scan kernels (inputs may be bf16 / fp16)

    def __init__(self, dtype=torch.float32):
        self.dtype = dtype
        self.esize = torch.finfo(dtype).bits // 8

    # --- to define per workload
    def make_host(self, rows: int, seed: int):  # -> (inputs, cotangents), fp32 CPU tensors
        raise NotImplementedError

    def forward(self, *inputs):
        raise NotImplementedError

    def cpu_step(self, sample):
        raise NotImplementedError

    # --- shared plumbing
    @property
    def elems(self) -> int:
        return self.B * self.T * self.D

    def host_inputs(self, rank: int):
        ins, cots = self.make_host(self.B, seed=rank)
        return [x.to(self.dtype) for x in ins], [c.to(self.dtype) for c in cots]

    def device_setup(self, host, dev):
        ins, cots = host
        return {"ins": [x.to(dev).requires_grad_(True) for x in ins],
                "cots": [c.to(dev) for c in cots]}

    def step(self, st, events=None):
        if events:
            events[0].record()
        outs = self.forward(*st["ins"])
        if events:
            events[1].record()
        grads = torch.autograd.grad(outs, st["ins"], st["cots"])
        if events:
            events[2].record()
        return outs, grads

    def e2e_setup(self, host, dev):
        ins, cots = host
        pins = [x.pin_memory() for x in ins]
        pcots = [c.pin_memory() for c in cots]
        outs = [torch.empty_like(c).pin_memory() for c in cots] + [torch.empty_like(x).pin_memory() for x in ins]
        # two device copies of a step's inputs, filled alternately (no allocation per step)
        slots = [([torch.empty_like(x, device=dev).requires_grad_(True) for x in ins],
                  [torch.empty_like(c, device=dev) for c in cots]) for _ in range(2)]
        return {"ins": pins, "cots": pcots, "out": outs, "dev": dev, "slots": slots}

    def e2e_h2d(self, st, slot):
        """One step's inputs and cotangents, copied from the pinned host buffers
        into device slot `slot`."""
        ins, cots = st["slots"][slot]
        with torch.no_grad():
            for d, h in zip(ins + cots, st["ins"] + st["cots"]):
                d.copy_(h, non_blocking=True)
        return ins, cots

    def e2e_compute(self, st, ins, cots):
        """The public op and its autograd backward: the step's results."""
        outs = self.forward(*ins)
        grads = torch.autograd.grad(outs, ins, cots)
        return list(outs) + list(grads)

    @property
    def footprint_bytes(self) -> int:
        """Bytes one fwd+bwd step touches (inputs, cotangents, outputs, grads)."""
        return int((self.fwd_bytes + self.bwd_bytes) * self.elems)

    def _bytes(self, tensors) -> int:
        return sum(t.numel() for t in tensors) * self.esize

    @property
    def h2d_bytes(self) -> int:
        ins, cots = self._shape_probe
        return self._bytes(ins) + self._bytes(cots)

    @property
    def d2h_bytes(self) -> int:
        ins, cots = self._shape_probe
        return self._bytes(cots) + self._bytes(ins)  # outputs (shaped like cots) + grads

    @property
    def _shape_probe(self):
        if not hasattr(self, "_probe"):
            ins, cots = self.make_host(self.B, seed=0)
            self._probe = ([torch.empty(x.shape, device="meta") for x in ins],
                           [torch.empty(c.shape, device="meta") for c in cots])
        return self._probe

    def cpu_sample(self, rows: int):
        ins, cots = self.make_host(rows, seed=0)
        return [x.numpy() for x in ins], [c.numpy() for c in cots]

    def sample_elems(self, rows: int) -> int:
        return rows * self.T * self.D

    def sample_desc(self, rows: int) -> str:
        return f"{rows} of {self.B} batch rows (T={self.T}, D={self.D})"

    def config(self, n_gpus: int) -> dict:
        return {
            "workload": self.workload,
            "B_per_gpu": self.B,
            "global_batch": self.B * n_gpus,
            "T": self.T,
            "D": self.D,
            "elem": self.metric_elems_doc,
            "input_dtype": str(self.dtype).replace("torch.", ""),
            "l2": (f"step footprint {self.footprint_bytes / 1e6:.0f} MB > 2 x 126 MB L2: no flush"
                   if self.footprint_bytes >= L2_FLUSH_THRESHOLD else
                   f"step footprint {self.footprint_bytes / 1e6:.0f} MB fits L2: each step timed "
                   "alone after writing a 256 MB buffer"),
            "parallelism": f"batch-sharded x{n_gpus}, no collective",
        }


class LinearScanWorkload(ScanWorkload):
    """SignedMinGRU linear_scan fwd+bwd, B=16, T=4096, D=1024.

    a = tanh(N(0,1)), b ~ N(0,1) (seed 0); upstream grads gBc ~ N(0,1)
    (seed 1234, the reference parity harness's cotangent seed) and gA = 0
    (h_0 = 0 in SignedMinGRU, so dL/dA = dL/dh * h_0 = 0).
    """

    kernels = {"fwd": "linear_scan_fwd", "bwd": "linear_scan_bwd"}

    def __init__(self, dtype=torch.float32, name="cfg2", B=16, T=4096, D=1024):
        super().__init__(dtype)
        self.B, self.T, self.D, self.name = B, T, D, name
        self.fwd_bytes = 4 * self.esize  # a, b read; A, Bc written
        self.bwd_bytes = 6 * self.esize  # a, b, gA, gBc read; da, db written
        self.workload = ("linear_scan fwd+bwd (SignedMinGRU scan, BASELINE config 2"
                         + ("" if dtype == torch.float32 else ", bf16 inputs / fp32 state") + ")")

    def make_host(self, rows, seed):
        g = torch.Generator().manual_seed(seed)
        a = torch.tanh(torch.randn(rows, self.T, self.D, generator=g))
        b = torch.randn(rows, self.T, self.D, generator=g)
        gB = torch.randn(rows, self.T, self.D, generator=torch.Generator().manual_seed(1234 + seed))
        return [a, b], [torch.zeros_like(a), gB]

    def forward(self, a, b):
        import mingru_b200 as mb

        return mb.linear_scan(a, b)

    def cpu_step(self, sample):
        from oracle import oracle

        (a, b), (gA, gB) = sample
        A, Bc = oracle.linear_scan(a, b, dtype=np.float32)
        oracle.linear_scan_bwd(a, A, Bc, gA, gB, dtype=np.float32)


class LogScanWorkload(ScanWorkload):
    """MinGRU parallel_scan_log fwd+bwd, B=8, T=1024, D=256.

    k, x ~ N(0,1); log_coeffs = -softplus(k); log_values = [log h0,
    -softplus(-k) + log_g(x)] with h0 = 0 taken as log(float32 tiny) (a finite
    numerically-zero state, as MinGRU clamps it); grad_h ~ N(0,1) (seed 1234).
    """

    kernels = {"fwd": "log_scan_fwd", "bwd": "log_scan_bwd"}
    workload = "parallel_scan_log fwd+bwd (MinGRU scan, BASELINE config 1)"

    def __init__(self, dtype=torch.float32, name="cfg1", B=8, T=1024, D=256):
        super().__init__(dtype)
        self.B, self.T, self.D, self.name = B, T, D, name
        self.fwd_bytes = 3 * self.esize  # lc, lv read; h written
        self.bwd_bytes = 5 * self.esize  # lc, lv, grad_h read; dlc, dlv written

    def make_host(self, rows, seed):
        g = torch.Generator().manual_seed(seed)
        k = torch.randn(rows, self.T, self.D, generator=g)
        x = torch.randn(rows, self.T, self.D, generator=g)
        log_g = torch.where(x >= 0, (x.clamp_min(0) + 0.5).log(), -torch.nn.functional.softplus(-x))
        lc = -torch.nn.functional.softplus(k)
        lh0 = torch.full((rows, 1, self.D), math.log(torch.finfo(torch.float32).tiny))
        lv = torch.cat([lh0, -torch.nn.functional.softplus(-k) + log_g], 1)
        gh = torch.randn(rows, self.T, self.D, generator=torch.Generator().manual_seed(1234 + seed))
        return [lc, lv], [gh]

    def forward(self, lc, lv):
        import mingru_b200 as mb

        return (mb.parallel_scan_log(lc, lv),)

    def cpu_step(self, sample):
        from oracle import oracle

        (lc, lv), (gh,) = sample
        oracle.parallel_scan_log(lc, lv, dtype=np.float32)
        oracle.parallel_scan_log_bwd(lc, lv, gh, dtype=np.float32)


class GateScanWorkload(LogScanWorkload):
    """BASELINE config 1's MinGRU scan fed from the pre-activations: the gate
    scan (coefficient prologue fused into the scan kernels) on k, x~ ~ N(0,1)
    and log h0 = log(float32 tiny), B=8, T=1024, D=256. Same algorithmic bytes
    as config 1 (fwd reads k, x~ and writes h; bwd reads k, x~, grad_h and writes
    dk, dx~). The unfused path -- softplus / log_g / cat in torch, then
    parallel_scan_log -- is timed in the same run for comparison."""

    kernels = {"fwd": "log_gate_scan_fwd", "bwd": "log_gate_scan_bwd"}
    workload = ("MinGRU gate scan fwd+bwd from pre-activations (BASELINE config 1 shape, "
                "prologue fused)")

    def make_host(self, rows, seed):
        g = torch.Generator().manual_seed(seed)
        k = torch.randn(rows, self.T, self.D, generator=g)
        x = torch.randn(rows, self.T, self.D, generator=g)
        lh0 = torch.full((rows, self.D), math.log(torch.finfo(torch.float32).tiny))
        gh = torch.randn(rows, self.T, self.D, generator=torch.Generator().manual_seed(1234 + seed))
        return [k, x, lh0], [gh]

    def forward(self, k, x, lh0):
        import mingru_b200 as mb

        return (mb.mingru_gate_scan(k, x, lh0),)

    def unfused_forward(self, k, x, lh0):
        import mingru_b200 as mb

        F = torch.nn.functional
        lc = -F.softplus(k)
        lv = torch.cat([lh0[:, None], -F.softplus(-k) + mb.log_g(x)], 1)
        return (mb.parallel_scan_log(lc, lv),)

    def cpu_step(self, sample):
        from oracle import oracle

        (k, x, lh0), (gh,) = sample
        lc, lv = oracle.mingru_gate_logs(k, x, lh0)
        oracle.parallel_scan_log(lc, lv, dtype=np.float32)
        oracle.parallel_scan_log_bwd(lc, lv, gh, dtype=np.float32)


class MatrixScanWorkload(ScanWorkload):
    """RotationMinGRU matrix_scan (2x2 blocks) fwd+bwd,
    B=16, T=2048, D=512 (n=256 blocks): M = sigmoid(N(0,1)) * R(theta),
    theta ~ U(-pi, pi), b ~ N(0,1); grad_Bc ~ N(0,1), grad_A = 0 (h0 fixed)."""

    kernels = {"fwd": "affine_scan_fwd", "bwd": "affine_scan_bwd"}
    workload = "matrix_scan 2x2 fwd+bwd (RotationMinGRU scan, BASELINE config 3)"
    metric_elems_doc = "B*T*D with D = 2n"

    def __init__(self, dtype=torch.float32, name="cfg3", B=16, T=2048, D=512):
        super().__init__(dtype)
        self.B, self.T, self.D, self.name = B, T, D, name
        # per element (half a block): fwd reads M (2) + b (1), writes A (2) + Bc (1)
        self.fwd_bytes = 6 * self.esize
        # bwd reads M, b, gA, gBc (6) and writes dM, db (3)
        self.bwd_bytes = 9 * self.esize

    def make_host(self, rows, seed):
        n = self.D // 2
        g = torch.Generator().manual_seed(seed)
        th = (torch.rand(rows, self.T, n, generator=g) * 2 - 1) * math.pi
        sc = torch.sigmoid(torch.randn(rows, self.T, n, generator=g))
        c, sn = torch.cos(th), torch.sin(th)
        M = sc[..., None, None] * torch.stack([torch.stack([c, -sn], -1), torch.stack([sn, c], -1)], -2)
        b = torch.randn(rows, self.T, n, 2, generator=g)
        gB = torch.randn(rows, self.T, n, 2, generator=torch.Generator().manual_seed(1234 + seed))
        return [M, b], [torch.zeros_like(M), gB]

    def forward(self, M, b):
        import mingru_b200 as mb

        return mb.matrix_scan(M, b)

    def cpu_step(self, sample):
        from oracle import oracle

        (M, b), (gA, gB) = sample
        A, Bc = oracle.matrix_scan(M, b, dtype=np.float32)
        oracle.matrix_scan_bwd(M, A, Bc, gA, gB, dtype=np.float32)


class AngleScanWorkload(ScanWorkload):
    """GivensMinGRU angle-fused scan fwd+bwd, B=8, T=4096,
    D=1024 (n=128 blocks of k=8), R=2 brick-wall rounds with the wrap-around
    plane (7, 0) angle fixed to 0, i.e. the 7 nearest-neighbour Givens
    rotations, theta ~ U(-pi, pi); gamma = sigmoid(N(0,1)) (decay on),
    b ~ N(0,1), h0 = 0; grad_h ~ N(0,1). The matrices are never built."""

    kernels = {"fwd": "angle_scan_fwd", "bwd": "angle_scan_bwd"}
    workload = "angle-fused Givens scan k=8 R=2 fwd+bwd (GivensMinGRU, BASELINE config 4)"
    metric_elems_doc = "B*T*D with D = n*k"

    def __init__(self, dtype=torch.float32, name="cfg4", B=8, T=4096, D=1024, k=8, R=2):
        super().__init__(dtype)
        self.B, self.T, self.D, self.k, self.R, self.name = B, T, D, k, R, name
        self.n = D // k
        # per block-step: fwd reads theta (R*k/2), gamma (1), b (k), writes h (k);
        # bwd reads theta, gamma, b, grad_h and writes dtheta, dgamma, db (h0/dh0 per lane only)
        na = R * k // 2
        self.fwd_bytes = (na + 1 + 2 * k) * self.esize / k
        self.bwd_bytes = (2 * na + 2 + 3 * k) * self.esize / k

    def make_host(self, rows, seed):
        g = torch.Generator().manual_seed(seed)
        n, k, R = self.n, self.k, self.R
        theta = (torch.rand(rows, self.T, n, R, k // 2, generator=g) * 2 - 1) * math.pi
        theta[:, :, :, 1, k // 2 - 1] = 0.0  # plane (k-1, 0) of the second rotation layer fixed: 7 live rotations
        gamma = torch.sigmoid(torch.randn(rows, self.T, n, generator=g))
        b = torch.randn(rows, self.T, n, k, generator=g)
        h0 = torch.zeros(rows, n, k)
        gh = torch.randn(rows, self.T, n, k, generator=torch.Generator().manual_seed(1234 + seed))
        return [theta, gamma, b, h0], [gh]

    def device_setup(self, host, dev):
        import mingru_b200 as mb

        st = super().device_setup(host, dev)
        self._const(dev)
        return st

    def _const(self, dev):
        import mingru_b200 as mb

        if getattr(self, "_dev", None) != dev:
            self._dev = dev
            self.scale = torch.ones(self.B, self.T, self.n, dtype=self.dtype, device=dev)
            self.meta = mb.brickwall_meta(self.R, self.k, dev)

    def forward(self, theta, gamma, b, h0):
        import mingru_b200 as mb

        self._const(theta.device)
        scale = self.scale if self.scale.shape[0] == theta.shape[0] else torch.ones(
            theta.shape[:3], dtype=theta.dtype, device=theta.device)
        return (mb.angle_scan_impl(theta, scale, gamma, b, h0, *self.meta,
                                   has_scale=0, has_decay=1),)

    def cpu_step(self, sample):
        import mingru_b200 as mb
        from oracle import oracle

        (theta, gamma, b, h0), (gh,) = sample
        perm, sgn, p2p = (x.numpy() for x in mb.brickwall_meta(self.R, self.k))
        scale = np.ones(theta.shape[:3], dtype=np.float32)
        kw = dict(has_scale=0, has_decay=1, dtype=np.float32)
        h = oracle.angle_scan(theta, scale, gamma, b, h0, perm, sgn, p2p, **kw)
        oracle.angle_scan_bwd(theta, scale, gamma, h0, h, gh, perm, sgn, p2p, **kw)


class DeltaWorkload(ScanWorkload):
    """DeltaMinGRU chunked-WY delta rule fwd+bwd, H=8 heads,
    d_k=d_v=64, chunk=64, nh=1, T=8192, B=8 per GPU. K ~ N(0,1) L2-normalised
    over d_k, V, Q ~ N(0,1), beta = sigmoid(N(0,1)), H0 = 0; bf16 inputs with an
    fp32 state (y in bf16, H_T fp32); grad_y ~ N(0,1), grad_H_T = 0."""

    kernels = {"fwd": "delta_fwd", "bwd": "delta_bwd"}
    workload = "DeltaMinGRU chunked-WY fwd+bwd (BASELINE config 5, bf16 in / fp32 state)"
    metric_elems_doc = "B*T*H*d_v"
    launches_per_step = 4  # forward prep + chain kernels, backward chain + gradient kernels
    compute_dtype = "bf16"  # tensor-core products (hi + lo split operands), fp32 accumulate / state

    def __init__(self, dtype=torch.bfloat16, name="cfg5", B=8, T=8192, H=8, d=64, chunk=64):
        super().__init__(dtype)
        if dtype != torch.bfloat16:  # fp32 inputs: three-level operands, fp32-grade products
            self.compute_dtype = "f32"
            self.workload = self.workload.replace("bf16 in", "fp32 in")
        self.B, self.T, self.H, self.d, self.chunk, self.name = B, T, H, d, chunk, name
        self.D = H * d  # elems = B*T*H*d_v
        e = self.esize
        # per (token, head): fwd reads Q, K, V (d each) + beta, writes y (d);
        # bwd reads Q, K, V, beta, dy and writes dQ, dK, dV, dbeta.
        self.fwd_bytes = (4 * d + 1) * e / d
        self.bwd_bytes = (7 * d + 2) * e / d

    @property
    def flops(self) -> float:
        """FLOPs of the reference chunked-WY algorithm per step: fwd 3.40 M and bwd
        8.90 M per (b, h, chunk)."""
        return (3.40e6 + 8.90e6) * self.B * self.H * (self.T // self.chunk)

    def make_host(self, rows, seed):
        g = torch.Generator().manual_seed(seed)
        H, T, d = self.H, self.T, self.d
        Q = torch.randn(rows, H, T, d, generator=g)
        K = torch.nn.functional.normalize(torch.randn(rows, H, T, 1, d, generator=g), dim=-1)
        V = torch.randn(rows, H, T, 1, d, generator=g)
        beta = torch.sigmoid(torch.randn(rows, H, T, 1, generator=g))
        gy = torch.randn(rows, H, T, d, generator=torch.Generator().manual_seed(1234 + seed))
        return [Q, K, V, beta], [gy, torch.zeros(rows, H, d, d)]

    def device_setup(self, host, dev):
        ins, cots = host
        st = {"ins": [x.to(dev).requires_grad_(True) for x in ins],
              "cots": [cots[0].to(dev), cots[1].to(dev, torch.float32)]}
        self.H0 = torch.zeros(self.B, self.H, self.d, self.d, device=dev)
        return st

    def forward(self, Q, K, V, beta):
        import mingru_b200 as mb

        H0 = self.H0 if self.H0.shape[0] == Q.shape[0] else torch.zeros(
            Q.shape[0], self.H, self.d, self.d, device=Q.device)
        return mb.delta_scan_impl(Q, K, V, beta, H0, chunk_size=self.chunk)

    def e2e_setup(self, host, dev):
        ins, cots = host
        st = super().e2e_setup((ins, [cots[0]]), dev)
        st["dHT"] = torch.zeros(self.B, self.H, self.d, self.d, device=dev)
        return st

    def e2e_compute(self, st, ins, cots):
        y, HT = self.forward(*ins)
        grads = torch.autograd.grad((y, HT), ins, (cots[0], st["dHT"]))
        return [y] + list(grads)

    @property
    def h2d_bytes(self) -> int:
        return int((self.fwd_bytes + self.esize) * self.elems)  # Q, K, V, beta, grad_y

    @property
    def d2h_bytes(self) -> int:
        return int((self.fwd_bytes) * self.elems)  # y, dQ, dK, dV, dbeta

    cpu_heads = 1  # the fp64 numpy oracle is slow: one head of one batch row per sample

    def cpu_sample(self, rows: int):
        (Q, K, V, beta), (gy, gHT) = self.make_host(rows, seed=0)
        h = self.cpu_heads
        return ([Q[:, :h].numpy(), K[:, :h].numpy(), V[:, :h].numpy(), beta[:, :h].numpy()],
                [gy[:, :h].numpy(), gHT[:, :h].numpy()])

    def sample_elems(self, rows: int) -> int:
        return rows * self.cpu_heads * self.T * self.d

    def sample_desc(self, rows: int) -> str:
        return f"{rows} batch row x {self.cpu_heads} of {self.H} heads (T={self.T}, d={self.d})"

    def cpu_step(self, sample):
        from oracle import delta_oracle

        (Q, K, V, beta), (gy, gHT) = sample
        H0 = np.zeros((Q.shape[0], Q.shape[1], self.d, self.d))
        delta_oracle.delta_forward(Q, K, V, beta, H0, self.chunk)
        delta_oracle.delta_backward(Q, K, V, beta, H0, gy, gHT, self.chunk)


class GatedDeltaWorkload(DeltaWorkload):
    """Config 5's delta rule with per-token decay active (the reference runs
    _forward_chunked_gated in eager torch only): log gamma = -lambda dt with
    lambda = softplus(0) per head and dt ~ U(0, 2). Same tensors and bytes as
    config 5 plus the (B, H, T) log decay read and its gradient written."""

    kernels = {"fwd": "delta_gated_fwd", "bwd": "delta_gated_bwd"}
    workload = "DeltaMinGRU chunked-WY with decay fwd+bwd (BASELINE config 5 shape, bf16 in)"
    compute_dtype = "f32"  # CUDA-core kernels, fp32 arithmetic

    def make_host(self, rows, seed):
        ins, cots = super().make_host(rows, seed)
        g = torch.Generator().manual_seed(100 + seed)
        lg = -math.log(2.0) * torch.rand(rows, self.H, self.T, generator=g) * 2
        return ins + [lg], cots

    def device_setup(self, host, dev):
        ins, cots = host
        st = {"ins": [x.to(dev).requires_grad_(True) for x in ins[:4]] +
                     [ins[4].to(dev, torch.float32).requires_grad_(True)],
              "cots": [cots[0].to(dev), cots[1].to(dev, torch.float32)]}
        self.H0 = torch.zeros(self.B, self.H, self.d, self.d, device=dev)
        return st

    def forward(self, Q, K, V, beta, lg):
        import mingru_b200 as mb

        H0 = self.H0 if self.H0.shape[0] == Q.shape[0] else torch.zeros(
            Q.shape[0], self.H, self.d, self.d, device=Q.device)
        return mb.delta_gated_scan_impl(Q, K, V, beta, H0, lg, chunk_size=self.chunk)

    def e2e_setup(self, host, dev):
        ins, cots = host
        st = ScanWorkload.e2e_setup(self, (ins[:4], [cots[0]]), dev)
        st["lg"] = ins[4].to(dev, torch.float32)
        st["dHT"] = torch.zeros(self.B, self.H, self.d, self.d, device=dev)
        return st

    def e2e_compute(self, st, ins, cots):
        y, HT = self.forward(*ins, st["lg"])
        grads = torch.autograd.grad((y, HT), ins, (cots[0], st["dHT"]))
        return [y] + list(grads)

    cpu_heads = 1

    def cpu_sample(self, rows: int):
        (Q, K, V, beta, lg), (gy, gHT) = self.make_host(rows, seed=0)
        h = self.cpu_heads
        return ([Q[:, :h].numpy(), K[:, :h].numpy(), V[:, :h].numpy(), beta[:, :h].numpy(),
                 lg[:, :h].numpy()], [gy[:, :h].numpy(), gHT[:, :h].numpy()])

    def cpu_step(self, sample):
        from oracle import delta_oracle

        (Q, K, V, beta, lg), (gy, gHT) = sample
        H0 = np.zeros((Q.shape[0], Q.shape[1], self.d, self.d))
        delta_oracle.gated_sequential_torch(Q, K, V, beta, H0, lg, gy, gHT)


WORKLOADS = {
    "cfg1": lambda: LogScanWorkload(),
    "cfg1-gate": lambda: GateScanWorkload(name="cfg1-gate"),
    "cfg2": lambda: LinearScanWorkload(),
    "cfg2-bf16": lambda: LinearScanWorkload(dtype=torch.bfloat16, name="cfg2-bf16"),
    "cfg3": lambda: MatrixScanWorkload(),
    "cfg4": lambda: AngleScanWorkload(),
    "cfg5": lambda: DeltaWorkload(),
    # BASELINE config 5's multi-GPU case: global batch 64 (with --scaling strong,
    # split 32 / 16 / 8 per GPU over 2 / 4 / 8 GPUs)
    "cfg5-b64": lambda: DeltaWorkload(B=64, name="cfg5-b64"),
    "cfg5-gated": lambda: GatedDeltaWorkload(name="cfg5-gated"),
    # config 5 shape with fp32 inputs (the module's default dtype): CUDA-core kernels
    "cfg5-fp32": lambda: DeltaWorkload(dtype=torch.float32, name="cfg5-fp32"),
}


# ----------------------------------------------------------------- clocks --


class ClockSampler:
    """nvidia-smi sampling of SM clocks / throttle reasons during the timed region.

    A reader thread timestamps every sample on arrival; ``mark_start`` /
    ``mark_stop`` bracket the timed region and only samples inside it count.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.t0 = self.t1 = None

    def __enter__(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self

        def reader():
            for line in self.proc.stdout:
                self.lines.append((time.time(), line))

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        deadline = time.time() + 5.0
        while not self.lines and time.time() < deadline:  # wait for the first sample
            time.sleep(0.02)
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_stop(self):
        self.t1 = time.time()

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.06)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, mx, reasons = [], 0.0, set()
        lo = self.t0 if self.t0 is not None else 0.0
        hi = (self.t1 if self.t1 is not None else time.time()) + 0.06
        for ts, line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                mx = max(mx, float(parts[2]))
                if not (lo <= ts <= hi):
                    continue
                sm.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ arms --


def dist_setup(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world: int, dev):
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[dev.index])


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def count_mgs_launches(fn, dev) -> int | None:
    """Kernel launches of this library (kernels in namespace mgs) in one call
    of fn, from the CUDA activity of torch.profiler; None if it is unavailable."""
    try:
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize(dev)
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize(dev)
        return sum(1 for ev in prof.events()
                   if ev.device_type is not None and "cuda" in str(ev.device_type).lower()
                   and "mgs::" in ev.name)
    except Exception:  # profiler unavailable
        return None


def host_threads() -> int:
    """All host cores this process may run on; also applied to the oracle and torch."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    from oracle import oracle

    n = oracle.set_threads(n)
    torch.set_num_threads(n)
    return n


def cpu_rows(w, requested: int) -> int:
    """Batch rows of one CPU sample; the same rule for the `cpu_baseline` leg
    and the `--impl reference` arm, so both time the same rows."""
    return max(1, min(w.B, requested))


def time_cpu_baseline(w, rows: int, reps: int = 3) -> dict:
    threads = host_threads()
    rows = cpu_rows(w, rows)
    sample = w.cpu_sample(rows)
    w.cpu_step(sample)  # warm-up (the first call also loads the oracle library)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        w.cpu_step(sample)
        times.append(time.perf_counter() - t0)
    dt = statistics.median(times)
    elems = w.sample_elems(rows)
    return {"value": elems / dt / 1e9, "unit": "Gelem/s", "cores": threads, "kind": "port",
            "sample": f"{w.sample_desc(rows)} fwd+bwd through the CPU oracle "
                      f"(restatement of the reference algorithm, {threads} threads), "
                      f"median of {reps} after 1 warm-up"}



def run_reference(args, w) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = host_threads()
    rows = cpu_rows(w, args.ref_rows)
    sample = w.cpu_sample(rows)
    for _ in range(args.warmup):
        w.cpu_step(sample)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        w.cpu_step(sample)
    dt = (time.perf_counter() - t0) / args.steps
    elems = w.sample_elems(rows)
    val = elems / dt / 1e9
    line = {
        "impl": "reference", "metric": "scan fwd+bwd Gelem/s", "value": val, "unit": "Gelem/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE shapes)",
        "config": w.config(args.gpus),
        "cpu_baseline": {"value": val, "unit": "Gelem/s", "cores": threads, "kind": "port",
                         "sample": f"{w.sample_desc(rows)} per step; CPU restatement of the "
                                   "reference algorithm (oracle/), "
                                   f"{threads} threads"},
        "e2e": {"value": val, "unit": "Gelem/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


REF_DIR = Path(__file__).resolve().parent / "baseline" / "_ref"


def ref_forward_fn(w, ref):
    """The reference's own GPU entry for this workload's op (its Triton kernels,
    MINGRU_SCAN=triton), taking the same arguments as `w.forward`; or the reason
    there is none. `ref` is the reference package."""
    ts = ref.triton_scans
    if isinstance(w, GateScanWorkload):
        return None, "the reference has no fused gate kernel (MinGRU builds its scan inputs in torch)"
    if isinstance(w, LogScanWorkload):
        return (lambda lc, lv: (ref.parallel_scan_log(lc, lv),)), None
    if isinstance(w, LinearScanWorkload):
        return ref.linear_scan, None
    if isinstance(w, MatrixScanWorkload):
        return ref.matrix_scan, None
    if isinstance(w, AngleScanWorkload):
        def angle(theta, gamma, b, h0):
            w._const(theta.device)
            return (ts.angle_scan_impl(theta, w.scale, gamma, b, h0, *w.meta,
                                       has_scale=0, has_decay=1),)
        return angle, None
    if isinstance(w, GatedDeltaWorkload):
        return None, "the reference runs the decay-active delta rule eagerly only (no kernel)"
    if isinstance(w, DeltaWorkload):
        if w.dtype != torch.float32:
            return None, "the reference's Triton delta kernel takes fp32 inputs only (use cfg5-fp32)"
        return (lambda Q, K, V, beta: ts.delta_scan_impl(Q, K, V, beta, w.H0,
                                                         chunk_size=w.chunk)), None
    return None, f"no reference GPU entry for {w.name}"


def run_reference_gpu(args, w) -> None:
    """The reference's own Triton kernels for the same op, inputs and step on
    this GPU (rank 0 only): its public op + autograd with MINGRU_SCAN=triton,
    from the reference package in baseline/_ref. Eager steps (the reference's
    ops launch from Python), each timed with CUDA events, median reported; each
    step alone after an L2 flush where the footprint fits L2, as for this
    library's line."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    base = {"impl": "reference-gpu", "metric": "scan fwd+bwd Gelem/s", "unit": "Gelem/s",
            "config": w.config(1)}
    os.environ["MINGRU_SCAN"] = "triton"
    if not (REF_DIR / "mingru").is_dir():
        print(json.dumps({**base, "unavailable": "reference package not in baseline/_ref"}))
        return
    sys.path.insert(0, str(REF_DIR))
    import mingru as ref
    import mingru.triton_scans  # noqa: F401  (the reference imports it lazily)

    ok = ref.triton_scans.available()
    if ok is not True:
        print(json.dumps({**base, "unavailable": f"reference Triton path unavailable: {ok}"}))
        return
    fwd, why = ref_forward_fn(w, ref)
    if fwd is None:
        print(json.dumps({**base, "unavailable": why}))
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    st = w.device_setup(w.host_inputs(0), dev)

    def step():
        outs = fwd(*st["ins"])
        return torch.autograd.grad(outs, st["ins"], st["cots"])

    for _ in range(args.warmup):  # the first call JIT-compiles the kernels
        step()
    torch.cuda.synchronize(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    flush = (torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
             if w.footprint_bytes < L2_FLUSH_THRESHOLD else None)
    for i, (a, b) in enumerate(evs):
        if flush is not None:
            flush.fill_(i & 255)
        a.record()
        step()
        b.record()
    torch.cuda.synchronize(dev)
    ms = statistics.median(a.elapsed_time(b) for a, b in evs)
    print(json.dumps({
        **base, "value": w.elems / (ms * 1e-3) / 1e9, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": w.compute_dtype, "data": "synthetic (seeded, BASELINE shapes)",
        "reference": f"mingru {ref.__version__} Triton kernels (MINGRU_SCAN=triton), "
                     "JIT-compiled for this GPU; median of per-step CUDA-event times",
    }), flush=True)


def capture(fn, dev, warm: int = 2, stream=None):
    """Capture fn() (a fixed sequence of launches on the current stream) in a CUDA graph."""
    side = stream if stream is not None else torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(warm):
            fn()
    torch.cuda.current_stream(dev).wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        keep = fn()
    return g, keep


def time_graph(g, reps: int, dev, flush=None) -> float:
    """Average device ms per replay of graph g (events on the replay stream);
    with `flush`, each replay is timed alone after overwriting L2."""
    g.replay()
    torch.cuda.synchronize(dev)
    if flush is not None:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(reps)]
        for i, (a, b) in enumerate(evs):
            flush.fill_(i & 255)
            a.record()
            g.replay()
            b.record()
        torch.cuda.synchronize(dev)
        return sum(a.elapsed_time(b) for a, b in evs) / reps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / reps


def gpu_numa_cpus(dev) -> tuple[int | None, set[int] | None]:
    """NUMA node of the GPU's PCIe device and that node's CPUs (None if unknown)."""
    try:
        pr = torch.cuda.get_device_properties(dev)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
    except AttributeError:
        return None, None
    try:
        node = int(Path(f"/sys/bus/pci/devices/{bus}/numa_node").read_text())
        if node < 0:
            return None, None
        cpus: set[int] = set()
        for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().split(","):
            lo, _, hi = part.strip().partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        return node, cpus & os.sched_getaffinity(0)
    except (OSError, ValueError):
        return None, None


class NumaLocal:
    """Run a block on the CPUs of the GPU's NUMA node, so the pinned host buffers
    it allocates (first touch) are local to the GPU's PCIe root; the previous
    affinity is restored afterwards."""

    def __init__(self, dev):
        self.node, self.cpus = gpu_numa_cpus(dev)
        self.saved = None

    def __enter__(self):
        if self.cpus:
            self.saved = os.sched_getaffinity(0)
            os.sched_setaffinity(0, self.cpus)
        return self

    def __exit__(self, *exc):
        if self.saved is not None:
            os.sched_setaffinity(0, self.saved)


def run_ours(args, w) -> None:
    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    import mingru_b200 as mb

    if args.scaling == "strong":  # the configuration's batch is the global batch
        if w.B % world:
            raise SystemExit(f"--scaling strong: global batch {w.B} does not split over {world} GPUs")
        w.global_B = w.B
        w.B //= world
    host = w.host_inputs(rank)
    # Every kernel of the run is issued on one stream: warm-up, graph capture,
    # the per-kernel graphs and the e2e compute (so each autograd leaf sees its
    # forward and backward on the same stream).
    work = torch.cuda.Stream(dev)
    with torch.cuda.stream(work):
        st = w.device_setup(host, dev)
        for _ in range(args.warmup):
            w.step(st)
        torch.cuda.synchronize(dev)
        mb.raise_device_error(dev)

        # One step = forward + backward of the op, replayed as a CUDA graph so
        # the device, not Python dispatch, sets the pace (every kernel of the
        # step runs on every replay; inputs stay resident in HBM).
        graph = None
        if not args.no_graph:
            graph, _keep = capture(lambda: w.step(st), dev, stream=work)

        # Inputs smaller than L2 would be served from cache on back-to-back
        # steps: then every step is timed alone, after writing a buffer larger
        # than L2.
        flush = None
        if w.footprint_bytes < L2_FLUSH_THRESHOLD:
            flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
        run_step = (graph.replay if graph is not None else (lambda: w.step(st)))

        def window() -> float:
            """Exactly `steps` steps bracketed by a barrier and a synchronize on
            both sides; device ms (max over ranks)."""
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)] if flush is not None else []
            barrier(world, dev)
            torch.cuda.synchronize(dev)
            start.record()
            for i in range(args.steps):
                if flush is not None:
                    flush.fill_(i & 255)
                    evs[i][0].record()
                run_step()
                if flush is not None:
                    evs[i][1].record()
            stop.record()
            torch.cuda.synchronize(dev)
            barrier(world, dev)
            local_ms = (sum(a.elapsed_time(b) for a, b in evs) if flush is not None
                        else start.elapsed_time(stop))
            return max_over_ranks(local_ms, world, dev)

        # Several windows of K steps each (enough for a few clock samples), the
        # median reported; every rank runs the same number of windows.
        with ClockSampler(dev.index) as clk:
            clk.mark_start()
            t0 = time.perf_counter()
            wins = [window()]
            first_s = time.perf_counter() - t0
            n_win = int(max_over_ranks(
                float(max(1, min(args.max_windows, math.ceil(args.min_seconds / max(first_s, 1e-4))))),
                world, dev))
            for _ in range(n_win - 1):
                wins.append(window())
            clk.mark_stop()
        ms = statistics.median(wins)
        mb.raise_device_error(dev)

        # Per-kernel device time: each op captured alone and replayed.
        ins, cots = st["ins"], st["cots"]
        with torch.no_grad():
            gf, _kf = capture(lambda: w.forward(*ins), dev, stream=work)
        outs = w.forward(*ins)
        gb, _kb = capture(lambda: torch.autograd.grad(outs, ins, cots, retain_graph=True), dev,
                          stream=work)
        reps = max(10, min(200, args.steps))
        fwd_ms = time_graph(gf, reps, dev, flush)
        bwd_ms = time_graph(gb, reps, dev, flush)
        del gf, gb, _kf, _kb, outs, graph
        unfused_ms = None
        if hasattr(w, "unfused_forward"):  # the same step through the unfused path
            def unfused_step():
                o = w.unfused_forward(*ins)
                return o, torch.autograd.grad(o, ins, cots)
            gu, _ku = capture(unfused_step, dev, stream=work)
            unfused_ms = time_graph(gu, reps, dev, flush)
            del gu, _ku

        # ---- e2e: public API with pinned host buffers, copies inside the timed region
        with NumaLocal(dev) as numa:
            est = w.e2e_setup(host, dev)
        e2e_pipeline(w, est, max(1, min(args.warmup, 3)), dev)
        torch.cuda.synchronize(dev)
        e_steps = max(1, min(args.steps, args.e2e_steps))
        barrier(world, dev)
        torch.cuda.synchronize(dev)
        e_ms = max_over_ranks(e2e_pipeline(w, est, e_steps, dev), world, dev)
        barrier(world, dev)

    cpu = (time_cpu_baseline(w, args.ref_rows)
           if (rank == 0 and world == 1 and not args.no_cpu) else None)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return

    peaks, peak_kind = load_peaks()
    traffic = load_traffic()
    per_step_ms = ms / args.steps
    total_elems = w.elems * world
    dom = "bwd" if bwd_ms >= fwd_ms else "fwd"
    dom_ms = bwd_ms if dom == "bwd" else fwd_ms
    dom_bytes = (w.bwd_bytes if dom == "bwd" else w.fwd_bytes) * w.elems
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    key = f"{w.kernels[dom]}:{w.name}"
    cfg = dict(w.config(world), step="cuda-graph replay" if not args.no_graph else "eager",
               windows=f"median of {len(wins)} windows of {args.steps} steps "
                       f"(window ms min/median/max {min(wins):.3f}/{ms:.3f}/{max(wins):.3f})",
               host_numa_node=numa.node)
    if args.scaling == "strong":
        cfg.update(global_batch=w.global_B, B_per_gpu=w.B,
                   parallelism=f"batch-sharded x{world} (global batch {w.global_B} split "
                               f"{w.B} per GPU), no collective")
    line = {
        "metric": "scan fwd+bwd Gelem/s",
        "value": total_elems * args.steps / (ms * 1e-3) / 1e9,
        "unit": "Gelem/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per_step_ms,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": w.compute_dtype,
        "data": "synthetic (seeded, BASELINE shapes)",
        "config": cfg,
        "tflops": (w.flops / (per_step_ms * 1e-3) / 1e12) if hasattr(w, "flops") else None,
        "kernel_ms": {"fwd": fwd_ms, "bwd": bwd_ms},
        "unfused_ms_per_step": unfused_ms,
        "roofline": {
            "bound": "hbm",
            "kernel": w.kernels[dom],
            "achieved": achieved,
            "peak": peaks["hbm_gbs"],
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / peaks["hbm_gbs"],
            "traffic": traffic[key] * w.elems if key in traffic else None,
            "algorithmic_bytes": dom_bytes,
        },
        "step_hbm_frac": (w.fwd_bytes + w.bwd_bytes) * w.elems / (per_step_ms * 1e-3) / 1e9
        / peaks["hbm_gbs"],
        "cpu_baseline": cpu,
        "e2e": {
            "value": total_elems * e_steps / (e_ms * 1e-3) / 1e9,
            "unit": "Gelem/s",
            "h2d_bytes_per_step": w.h2d_bytes,
            "d2h_bytes_per_step": w.d2h_bytes,
            "path": "public op + autograd (C ABI) from pinned host buffers (allocated on the "
                    "GPU's NUMA node), eager; each step's host-to-device copy, compute and "
                    "device-to-host copy on three streams, so one step's inputs cross PCIe while "
                    "the previous step's results come back",
        },
        "gpu_launches": w.launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_stack(args) -> None:
    """MinGRUStack training step (forward, backward, AdamW) under a CUDA graph.

    Not a BASELINE configuration: it measures whether the scan kernels still
    dominate a whole training step once they are fast (the stack's LayerNorms,
    projections, MLPs and the optimizer around them). Synthetic input and a
    mean-square loss on the output; the step is captured once and replayed.
    Reports tokens/s of the graph replay, the eager step for comparison, and the
    share of the step's device time spent in this library's scan kernels
    (torch.profiler over replays, kernels named mgs::...)."""
    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    import mingru_b200 as mb

    B, T, D, L = args.stack_batch, args.stack_t, args.stack_d, args.stack_layers
    mixers = args.stack_mixers.split(",")
    mixers = (mixers * L)[:L]
    torch.manual_seed(0)
    model = mb.MinGRUStack(D, D, L, mixer=mixers).to(dev)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, capturable=True, foreach=True)
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(B, T, D, device=dev, generator=g)

    def step():
        opt.zero_grad(set_to_none=True)
        out, _ = model(x)
        loss = out.float().pow(2).mean()
        loss.backward()
        opt.step()
        return loss

    work = torch.cuda.Stream(dev)
    work.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(work):
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(dev)
        mb.raise_device_error(dev)
        # eager step time (for the graph's launch-overhead saving)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize(dev)
        eager_ms = e0.elapsed_time(e1) / args.steps
        graph = torch.cuda.CUDAGraph()
        opt.zero_grad(set_to_none=True)
        with torch.cuda.graph(graph, stream=work):
            static_loss = step()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize(dev)

        def window() -> float:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier(world, dev)
            torch.cuda.synchronize(dev)
            a.record()
            for _ in range(args.steps):
                graph.replay()
            b.record()
            torch.cuda.synchronize(dev)
            barrier(world, dev)
            return max_over_ranks(a.elapsed_time(b), world, dev)

        with ClockSampler(dev.index) as clk:
            clk.mark_start()
            t0 = time.perf_counter()
            wins = [window()]
            n_win = int(max_over_ranks(float(max(1, min(args.max_windows, math.ceil(
                args.min_seconds / max(time.perf_counter() - t0, 1e-4))))), world, dev))
            for _ in range(n_win - 1):
                wins.append(window())
            clk.mark_stop()
        ms = statistics.median(wins)
        mb.raise_device_error(dev)
        loss_val = float(static_loss.item())

        # device-time share of the scan kernels over a few replays
        share, scan_ms, kernels, n_mgs = None, None, {}, 0
        reps = 5
        try:
            from torch.profiler import ProfilerActivity, profile

            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                for _ in range(reps):
                    graph.replay()
                torch.cuda.synchronize(dev)
            tot = scan = 0.0
            for ev in prof.events():
                if ev.device_type is None or "cuda" not in str(ev.device_type).lower():
                    continue
                t = ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total
                tot += t
                if "mgs::" in ev.name:
                    n_mgs += 1
                    scan += t
                    short = ev.name.split("(")[0].replace("void ", "")
                    kernels[short] = kernels.get(short, 0.0) + t / reps / 1e3
            if tot > 0:
                share, scan_ms = scan / tot, scan / reps / 1e3
        except Exception as exc:  # profiler unavailable: report without the share
            kernels = {"profiler_error": str(exc)[:200]}
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return
    per_step = ms / args.steps
    line = {
        "metric": "MinGRUStack training step tokens/s",
        "value": B * T * world * args.steps / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded), random-init weights",
        "config": {"workload": "MinGRUStack fwd+bwd+AdamW step (CUDA graph)", "B_per_gpu": B,
                   "T": T, "d_model": D, "n_layers": L, "mixers": mixers,
                   "projections": "tf32" if args.tf32 else "fp32",
                   "windows": f"median of {len(wins)} windows of {args.steps} steps"},
        "eager_ms_per_step": eager_ms,
        "graph_speedup": eager_ms / per_step,
        "scan_share": share,
        "scan_ms_per_step": scan_ms,
        "scan_kernels_ms": kernels,
        "loss": loss_val,
        "gpu_launches": (n_mgs // reps) * args.steps if n_mgs else None,  # one timed window
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_sp(args) -> None:
    """Sequence-parallel scan on one GPU, the time axis cut into --sp-slices
    slices and every slice's per-rank work run in turn (carry summaries, the
    prefix / suffix composition of the gathered summaries, the scans from the
    carried-in states), the all-gathers replaced by stacking. Reports the whole
    sequence's fwd+bwd time through the sliced path next to the one-launch
    scan, i.e. what sequence parallelism costs in kernel work before any
    NCCL time (config 2 shape for linear_scan, config 1 for parallel_scan_log)."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    import mingru_b200 as mb
    from mingru_b200.parallel import (KernelOps, linear_prefix, linear_suffix, log_prefix,
                                      log_suffix)

    n = args.sp_slices
    ops = KernelOps()
    g = torch.Generator(device=dev).manual_seed(0)
    if args.config == "cfg2-sp":
        B, T, D = 16, 4096, 1024
        a = torch.tanh(torch.randn(B, T, D, device=dev, generator=g))
        b = torch.randn(B, T, D, device=dev, generator=g)
        gA = torch.zeros(B, T, D, device=dev)
        gB = torch.randn(B, T, D, device=dev, generator=g)
        per = T // n
        sl = [slice(r * per, (r + 1) * per) for r in range(n)]
        ta, tb = a.clone().requires_grad_(True), b.clone().requires_grad_(True)

        def plain():
            A, Bc = mb.linear_scan(ta, tb)
            return torch.autograd.grad((A, Bc), (ta, tb), (gA, gB))

        # each emulated rank holds its slice contiguously, as a real rank would
        al, bl, gAl, gBl = ([x[:, s].contiguous() for s in sl] for x in (a, b, gA, gB))

        def sliced():
            G = torch.stack([ops.linear_carry_fwd(al[r], bl[r]) for r in range(n)])
            outs = [ops.linear_fwd_fixup(al[r], bl[r], linear_prefix(G, r)) for r in range(n)]
            R = torch.stack([ops.linear_carry_bwd(al[r], gAl[r], gBl[r]) for r in range(n)])
            return [ops.linear_bwd_fixup(al[r], bl[r], outs[r][2], linear_suffix(R, r), gAl[r],
                                         gBl[r]) for r in range(n)]
        workload, nbytes = "linear_scan fwd+bwd, config 2 shape", 40 * B * T * D
    else:
        B, T, D = 8, 1024 * n, 256
        k = torch.randn(B, T, D, device=dev, generator=g)
        lc = -torch.nn.functional.softplus(k)
        lv = torch.cat([torch.full((B, 1, D), -87.0, device=dev),
                        -torch.nn.functional.softplus(-k) + mb.log_g(torch.randn(B, T, D, device=dev, generator=g))], 1)
        gh = torch.randn(B, T, D, device=dev, generator=g)
        per = T // n
        sl = [slice(r * per, (r + 1) * per) for r in range(n)]
        tlc, tlv = lc.clone().requires_grad_(True), lv.clone().requires_grad_(True)

        def plain():
            h = mb.parallel_scan_log(tlc, tlv)
            return torch.autograd.grad(h, (tlc, tlv), gh)

        # each emulated rank holds its slice contiguously, as a real rank would
        lcl = [lc[:, s].contiguous() for s in sl]
        lvl = [lv[:, s.start:s.stop + 1].contiguous() for s in sl]
        ghl = [gh[:, s].contiguous() for s in sl]

        def sliced():
            G = torch.stack([torch.cat([ops.log_carry_fwd(lcl[r], lvl[r]), lvl[r][:, 0].float()[None]])
                             for r in range(n)])
            outs = []
            for r in range(n):
                lh = log_prefix(G, r)
                outs.append((lh,) + tuple(ops.log_fwd_fixup(lcl[r], lvl[r], lh)))
            R = torch.stack([ops.log_carry_bwd(lcl[r], ghl[r]) for r in range(n)])
            return [ops.log_bwd_fixup(lcl[r], lvl[r], outs[r][0], outs[r][2], log_suffix(R, r),
                                      ghl[r]) for r in range(n)]
        workload, nbytes = f"parallel_scan_log fwd+bwd, config 1 shape x{n} in T", 32 * B * T * D
    work = torch.cuda.Stream(dev)
    work.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(work):
        for _ in range(args.warmup):
            plain()
            sliced()
        gp, _kp = capture(plain, dev, stream=work)
        gs, _ks = capture(sliced, dev, stream=work)
        reps = max(10, args.steps)
        per_sliced = count_mgs_launches(gs.replay, dev)
        with ClockSampler(dev.index) as clk:
            clk.mark_start()
            plain_ms = time_graph(gp, reps, dev)
            sliced_ms = time_graph(gs, reps, dev)
            clk.mark_stop()
        mb.raise_device_error(dev)
    elems = B * T * D
    peaks, peak_kind = load_peaks()
    line = {
        "metric": "scan fwd+bwd Gelem/s, sequence-parallel slices on one GPU",
        "value": elems / (sliced_ms * 1e-3) / 1e9,
        "unit": "Gelem/s",
        "n_gpus": 1,
        "steps": reps,
        "warmup": args.warmup,
        "ms_per_step": sliced_ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": {"workload": workload, "B": B, "T": T, "D": D, "slices": n,
                   "collectives": "none (all-gathers replaced by stacking on one GPU)"},
        "one_launch_ms_per_step": plain_ms,
        "one_launch_value": elems / (plain_ms * 1e-3) / 1e9,
        "sliced_over_one_launch": sliced_ms / plain_ms,
        "step_hbm_frac_one_launch": nbytes / (plain_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
        "gpu_launches": per_sliced * reps if per_sliced else None,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_sp_dist(args) -> None:
    """Sequence parallelism across GPUs (torchrun, one rank per GPU): rank r
    holds time slice r of a sequence N times the configuration's length (the
    config 2 shape per rank for cfg2-sp, config 1 for cfg1-sp: weak scaling in
    T), and one step is the public sp_* op forward + backward with its NCCL
    all-gathers. Timed eagerly with CUDA events, max over ranks; next to it each
    rank's plain one-launch scan of its own slice (what the slice costs
    without sequence parallelism)."""
    import torch.distributed as dist

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    import mingru_b200 as mb
    from mingru_b200.parallel import sp_linear_scan, sp_parallel_scan_log

    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    if args.config == "cfg2-sp":
        B, Tl, D = 16, 4096, 1024
        a = torch.tanh(torch.randn(B, Tl, D, device=dev, generator=g)).requires_grad_(True)
        b = torch.randn(B, Tl, D, device=dev, generator=g).requires_grad_(True)
        gA = torch.zeros(B, Tl, D, device=dev)
        gB = torch.randn(B, Tl, D, device=dev, generator=g)

        def sp_step():
            A, Bc = sp_linear_scan(a, b)
            return torch.autograd.grad((A, Bc), (a, b), (gA, gB))

        def plain_step():
            A, Bc = mb.linear_scan(a, b)
            return torch.autograd.grad((A, Bc), (a, b), (gA, gB))
        workload, per_elem = "linear_scan fwd+bwd, config 2 shape per rank, T split over ranks", 40
    else:
        B, Tl, D = 8, 1024, 256
        k = torch.randn(B, Tl, D, device=dev, generator=g)
        lc = (-torch.nn.functional.softplus(k)).requires_grad_(True)
        lv = torch.cat([torch.full((B, 1, D), -87.0, device=dev),
                        -torch.nn.functional.softplus(-k)
                        + mb.log_g(torch.randn(B, Tl, D, device=dev, generator=g))], 1).requires_grad_(True)
        gh = torch.randn(B, Tl, D, device=dev, generator=g)

        def sp_step():
            h = sp_parallel_scan_log(lc, lv)
            return torch.autograd.grad(h, (lc, lv), gh)

        def plain_step():
            h = mb.parallel_scan_log(lc, lv)
            return torch.autograd.grad(h, (lc, lv), gh)
        workload, per_elem = "parallel_scan_log fwd+bwd, config 1 shape per rank, T split over ranks", 32

    def timed(fn, steps):
        barrier(world, dev)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        barrier(world, dev)
        return max_over_ranks(e0.elapsed_time(e1) / steps, world, dev)

    for _ in range(args.warmup):
        sp_step()
        plain_step()
    per_sp = count_mgs_launches(sp_step, dev)
    steps = max(3, args.steps)
    with ClockSampler(dev.index) as clk:
        clk.mark_start()
        sp_ms = timed(sp_step, steps)
        clk.mark_stop()
    plain_ms = timed(plain_step, steps)
    mb.raise_device_error(dev)
    elems = B * Tl * D * world
    peaks, _ = load_peaks()
    if rank == 0:
        line = {
            "metric": "scan fwd+bwd Gelem/s, sequence-parallel over GPUs",
            "value": elems / (sp_ms * 1e-3) / 1e9,
            "unit": "Gelem/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": args.warmup,
            "ms_per_step": sp_ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded per rank)",
            "config": {"workload": workload, "B": B, "T_per_rank": Tl, "T_total": Tl * world,
                       "D": D, "parallelism": f"sp{world}", "step": "eager, public sp_* op + autograd",
                       "collectives": "NCCL all-gather of per-slice carries, forward and backward"},
            "local_one_launch_ms_per_step": plain_ms,
            "sp_over_local_one_launch": sp_ms / plain_ms,
            "step_hbm_frac_per_gpu": per_elem * B * Tl * D / (sp_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
            "gpu_launches": per_sp * steps if per_sp else None,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_stack_step(args) -> None:
    """MinGRUStack.step (the streaming / decoding path, one token per call for
    a batch of streams): tokens/s of the eager step loop and of the step
    captured once as a CUDA graph and replayed (state carried in static
    buffers). The mixers' recurrence updates are the fused step kernels."""
    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    import mingru_b200 as mb

    B, D, L = args.stack_batch, args.stack_d, args.stack_layers
    mixers = (args.stack_mixers.split(",") * L)[:L]
    torch.manual_seed(0)
    model = mb.MinGRUStack(D, D, L, mixer=mixers).to(dev).eval()
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(B, D, device=dev, generator=g)
    work = torch.cuda.Stream(dev)
    work.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(work), torch.no_grad():
        _, state = model.step(x, model.init_state())  # materialise every layer's state
        for _ in range(args.warmup):
            _, state = model.step(x, state)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            _, state = model.step(x, state)
        e1.record()
        torch.cuda.synchronize(dev)
        eager_ms = e0.elapsed_time(e1) / args.steps
        static = [s_.clone() for s_ in state]
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=work):
            out, new = model.step(x, static)
            for dst, src in zip(static, new):
                dst.copy_(src)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize(dev)
        per_token = count_mgs_launches(graph.replay, dev)
        with ClockSampler(dev.index) as clk:
            clk.mark_start()
            wins = []
            for _ in range(max(1, args.max_windows // 5)):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                barrier(world, dev)
                torch.cuda.synchronize(dev)
                a.record()
                for _ in range(args.steps):
                    graph.replay()
                b.record()
                torch.cuda.synchronize(dev)
                wins.append(max_over_ranks(a.elapsed_time(b), world, dev))
            clk.mark_stop()
        ms = statistics.median(wins)
        mb.raise_device_error(dev)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return
    per_tok = ms / args.steps
    line = {
        "metric": "MinGRUStack.step tokens/s (streaming decode)",
        "value": B * world * args.steps / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per_tok,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded), random-init weights",
        "config": {"workload": "MinGRUStack.step, one token per stream (CUDA graph)",
                   "streams_per_gpu": B, "d_model": D, "n_layers": L, "mixers": mixers,
                   "projections": "tf32" if args.tf32 else "fp32",
                   "windows": f"median of {len(wins)} windows of {args.steps} steps"},
        "eager_ms_per_step": eager_ms,
        "graph_speedup": eager_ms / per_tok,
        "gpu_launches": per_token * args.steps if per_token else None,  # one timed window
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def e2e_pipeline(w, est, steps: int, dev) -> float:
    """Run `steps` end-to-end steps and return their device time in ms.

    Step k copies its inputs in on one stream, runs the public op and its
    backward on the current stream once they have landed, and copies its
    results out to the pinned host buffers on a third stream once they are
    computed. PCIe carries both directions at once, so step k+1's inputs
    travel while step k computes and step k-1's results come back. Inputs
    land in two preallocated device slots, used alternately: slot k % 2 is
    refilled once step k - 2's compute is done with it. The events bracket
    all three streams."""
    cs = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cs)
    s_in.wait_stream(cs)
    s_out.wait_stream(cs)
    done = []
    for k in range(steps):
        if k >= 2:
            s_in.wait_event(done[k - 2])
        with torch.cuda.stream(s_in):
            ins, cots = w.e2e_h2d(est, k % 2)
        cs.wait_stream(s_in)
        res = w.e2e_compute(est, ins, cots)
        ev = torch.cuda.Event()
        ev.record(cs)
        done.append(ev)
        s_out.wait_event(ev)
        with torch.cuda.stream(s_out):
            for o, r in zip(est["out"], res):
                o.copy_(r.detach(), non_blocking=True)
        for r in res:
            r.record_stream(s_out)
        del ins, cots, res
    cs.wait_stream(s_in)
    cs.wait_stream(s_out)
    e1.record(cs)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-gpu"], default="ours",
                    help="reference: the reference's CPU path (the oracle port); reference-gpu: "
                         "the reference's own Triton kernels on this GPU, if baseline/_ref holds it")
    ap.add_argument("--config", choices=sorted(WORKLOADS) + ["stack", "stack-step", "cfg1-sp",
                                                              "cfg2-sp"],
                    default="cfg2")
    ap.add_argument("--sp-slices", type=int, default=4,
                    help="cfg1-sp / cfg2-sp: time slices (emulated ranks) on one GPU")
    ap.add_argument("--stack-batch", type=int, default=8)
    ap.add_argument("--stack-t", type=int, default=1024)
    ap.add_argument("--stack-d", type=int, default=512)
    ap.add_argument("--stack-layers", type=int, default=4)
    ap.add_argument("--tf32", action="store_true",
                    help="stack benches: let torch run the fp32 projections on TF32 tensor cores "
                         "(default: exact fp32, as torch and the reference default to)")
    ap.add_argument("--stack-mixers", default="log,signed,rotation,givens",
                    help="comma-separated mixers, cycled over the layers")
    ap.add_argument("--e2e-steps", type=int, default=20,
                    help="steps of the e2e pipeline (at most --steps); the first step's copy-in "
                         "and the last step's copy-out overlap nothing, so few steps understate "
                         "the steady state")
    ap.add_argument("--ref-rows", type=int, default=2,
                    help="batch rows of each CPU sample (reference arm and cpu_baseline)")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="weak: the configuration's batch on every GPU; strong: it is the global "
                         "batch, split over the GPUs")
    ap.add_argument("--min-seconds", type=float, default=0.5,
                    help="time windows of --steps steps until about this long has run")
    ap.add_argument("--max-windows", type=int, default=50)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-graph", action="store_true", help="time eager steps instead of graph replay")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the per-GPU batch (small ncu captures only; not a bench line)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # timing rule: at least 3 untimed warm-up steps
    if args.config in ("cfg1-sp", "cfg2-sp"):
        if args.impl != "ours":
            print(json.dumps({"impl": args.impl, "unavailable": "the sliced scan has no "
                              "reference arm (the reference arms time the scan path)"}))
            return
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            run_sp_dist(args)
        else:
            run_sp(args)
        return
    if args.config in ("stack", "stack-step"):
        if args.impl != "ours":
            print(json.dumps({"impl": args.impl, "unavailable": "the stack benches have no "
                              "reference arm (the reference arms time the scan path)"}))
            return
        torch.backends.cuda.matmul.allow_tf32 = args.tf32
        torch.backends.cudnn.allow_tf32 = args.tf32
        (run_stack if args.config == "stack" else run_stack_step)(args)
        return
    w = WORKLOADS[args.config]()
    if args.batch is not None:
        w.B = args.batch
    if args.impl == "reference":
        run_reference(args, w)
    elif args.impl == "reference-gpu":
        run_reference_gpu(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
