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


class LinearScanWorkload:
    """SignedMinGRU linear_scan fwd+bwd.

    a = tanh(N(0,1)), b ~ N(0,1) (seed 0); upstream grads gBc ~ N(0,1)
    (seed 1234, the reference parity harness's cotangent seed) and gA = 0
    (h_0 = 0 in SignedMinGRU, so dL/dA = dL/dh * h_0 = 0).
    """

    def __init__(self, B=16, T=4096, D=1024, dtype=torch.float32, name="cfg2"):
        self.B, self.T, self.D, self.dtype, self.name = B, T, D, dtype, name
        self.esize = torch.finfo(dtype).bits // 8
        # algorithmic bytes per element: fwd reads a, b and writes A, Bc;
        # bwd reads a, b, gA, gBc and writes da, db.
        self.fwd_bytes = 4 * self.esize
        self.bwd_bytes = 6 * self.esize
        self.kernels = {"fwd": "linear_scan_fwd", "bwd": "linear_scan_bwd"}

    @property
    def elems(self) -> int:
        return self.B * self.T * self.D

    def config(self, n_gpus: int) -> dict:
        return {
            "workload": f"linear_scan fwd+bwd (SignedMinGRU scan, BASELINE config 2"
            f"{'' if self.dtype == torch.float32 else ', bf16 inputs / fp32 state'})",
            "B_per_gpu": self.B,
            "global_batch": self.B * n_gpus,
            "T": self.T,
            "D": self.D,
            "input_dtype": str(self.dtype).replace("torch.", ""),
            "l2": f"inputs {self.elems * self.esize / 1e6:.0f} MB each > 126 MB L2; no flush",
            "parallelism": f"batch-sharded x{n_gpus}, no collective",
        }

    def host_inputs(self, rank: int):
        g = torch.Generator().manual_seed(rank)
        a = torch.tanh(torch.randn(self.B, self.T, self.D, generator=g))
        b = torch.randn(self.B, self.T, self.D, generator=g)
        gB = torch.randn(self.B, self.T, self.D, generator=torch.Generator().manual_seed(1234 + rank))
        gA = torch.zeros(self.B, self.T, self.D)
        return [x.to(self.dtype) for x in (a, b, gA, gB)]

    def device_setup(self, host, dev):
        a, b, gA, gB = (x.to(dev) for x in host)
        return {"a": a.requires_grad_(True), "b": b.requires_grad_(True), "gA": gA, "gB": gB}

    def step(self, st, events=None):
        import mingru_b200 as mb

        if events:
            events[0].record()
        A, Bc = mb.linear_scan(st["a"], st["b"])
        if events:
            events[1].record()
        da, db = torch.autograd.grad((A, Bc), (st["a"], st["b"]), (st["gA"], st["gB"]))
        if events:
            events[2].record()
        return A, Bc, da, db

    launches_per_step = 2  # linear_scan fwd kernel + bwd kernel

    def e2e_setup(self, host, dev):
        pinned = [x.pin_memory() for x in host]
        outs = [torch.empty_like(pinned[0]).pin_memory() for _ in range(4)]
        return {"host": pinned, "out": outs, "dev": dev}

    def e2e_step(self, st):
        import mingru_b200 as mb

        dev = st["dev"]
        a, b, gA, gB = (x.to(dev, non_blocking=True) for x in st["host"])
        a.requires_grad_(True)
        b.requires_grad_(True)
        A, Bc = mb.linear_scan(a, b)
        da, db = torch.autograd.grad((A, Bc), (a, b), (gA, gB))
        for o, r in zip(st["out"], (A, Bc, da, db)):
            o.copy_(r.detach(), non_blocking=True)

    @property
    def h2d_bytes(self) -> int:
        return 4 * self.elems * self.esize

    @property
    def d2h_bytes(self) -> int:
        return 4 * self.elems * self.esize

    # --- CPU baseline: the oracle port of the reference algorithm (fp32 C, OpenMP)
    def cpu_sample(self, rows: int):
        g = torch.Generator().manual_seed(0)
        a = torch.tanh(torch.randn(rows, self.T, self.D, generator=g)).numpy()
        b = torch.randn(rows, self.T, self.D, generator=g).numpy()
        gB = torch.randn(rows, self.T, self.D, generator=g).numpy()
        return a, b, np.zeros_like(a), gB

    def cpu_step(self, sample):
        from oracle import oracle

        a, b, gA, gB = sample
        A, Bc = oracle.linear_scan(a, b, dtype=np.float32)
        oracle.linear_scan_bwd(a, A, Bc, gA, gB, dtype=np.float32)


WORKLOADS = {
    "cfg2": lambda: LinearScanWorkload(),
    "cfg2-bf16": lambda: LinearScanWorkload(dtype=torch.bfloat16, name="cfg2-bf16"),
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


def time_cpu_baseline(w, target_s: float = 12.0) -> dict:
    threads = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    rows = 1
    sample = w.cpu_sample(rows)
    t0 = time.perf_counter()
    w.cpu_step(sample)
    one = time.perf_counter() - t0
    rows = int(max(1, min(w.B, target_s / max(one, 1e-3) / 2)))
    sample = w.cpu_sample(rows)
    w.cpu_step(sample)  # warm-up
    times = []
    for _ in range(2):
        t0 = time.perf_counter()
        w.cpu_step(sample)
        times.append(time.perf_counter() - t0)
    dt = min(times)
    elems = rows * w.T * w.D
    return {"value": elems / dt / 1e9, "unit": "Gelem/s", "cores": threads, "kind": "port",
            "sample": f"{rows} of {w.B} batch rows (T={w.T}, D={w.D}) fwd+bwd, fp32 C oracle "
                      f"(OpenMP {threads} threads), best of 2 after 1 warm-up"}


def run_reference(args, w) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    rows = max(1, min(w.B, args.ref_rows))
    sample = w.cpu_sample(rows)
    for _ in range(args.warmup):
        w.cpu_step(sample)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        w.cpu_step(sample)
    dt = (time.perf_counter() - t0) / args.steps
    elems = rows * w.T * w.D
    val = elems / dt / 1e9
    line = {
        "impl": "reference", "metric": "scan fwd+bwd Gelem/s", "value": val, "unit": "Gelem/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE shapes)",
        "config": w.config(args.gpus),
        "cpu_baseline": {"value": val, "unit": "Gelem/s", "cores": threads, "kind": "port",
                         "sample": f"{rows} of {w.B} batch rows per step (T={w.T}, D={w.D}); "
                                   "sequential fp32 C restatement of the reference algorithm "
                                   f"(oracle/scan_oracle.c), OpenMP {threads} threads"},
        "e2e": {"value": val, "unit": "Gelem/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, w) -> None:
    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    import mingru_b200 as mb

    host = w.host_inputs(rank)
    st = w.device_setup(host, dev)
    for _ in range(args.warmup):
        w.step(st)
    torch.cuda.synchronize(dev)
    mb.raise_device_error(dev)

    # ---- timed region: device-resident inputs
    n_ev = args.steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n_ev)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world, dev)
    torch.cuda.synchronize(dev)
    with ClockSampler(dev.index) as clk:
        clk.mark_start()
        start.record()
        for i in range(args.steps):
            w.step(st, evs[i])
        stop.record()
        torch.cuda.synchronize(dev)
        clk.mark_stop()
    barrier(world, dev)
    ms = max_over_ranks(start.elapsed_time(stop), world, dev)
    mb.raise_device_error(dev)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)

    # ---- e2e: public API with pinned host buffers, copies inside the timed region
    est = w.e2e_setup(host, dev)
    for _ in range(max(1, min(args.warmup, 3))):
        w.e2e_step(est)
    torch.cuda.synchronize(dev)
    e_steps = max(1, min(args.steps, args.e2e_steps))
    barrier(world, dev)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e_steps):
        w.e2e_step(est)
    e1.record()
    torch.cuda.synchronize(dev)
    barrier(world, dev)
    e_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)

    cpu = time_cpu_baseline(w) if (rank == 0 and world == 1 and not args.no_cpu) else None
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return

    peaks, peak_kind = load_peaks()
    traffic = load_traffic()
    per_step_ms = ms / args.steps
    total_elems = w.elems * world
    # dominant kernel: the one with the larger share of the step
    dom = "bwd" if bwd_ms >= fwd_ms else "fwd"
    dom_ms = bwd_ms if dom == "bwd" else fwd_ms
    dom_bytes = (w.bwd_bytes if dom == "bwd" else w.fwd_bytes) * w.elems
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    key = f"{w.kernels[dom]}:{w.name}"
    line = {
        "metric": "scan fwd+bwd Gelem/s",
        "value": total_elems * args.steps / (ms * 1e-3) / 1e9,
        "unit": "Gelem/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": per_step_ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded, BASELINE shapes)",
        "config": w.config(world),
        "kernel_ms": {"fwd": fwd_ms, "bwd": bwd_ms},
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
            "path": "mingru_b200.linear_scan + autograd (C ABI) from pinned host buffers",
        },
        "gpu_launches": w.launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(WORKLOADS), default="cfg2")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--ref-rows", type=int, default=2, help="batch rows per reference step")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the per-GPU batch (small ncu captures only; not a bench line)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # timing rule: at least 3 untimed warm-up steps
    w = WORKLOADS[args.config]()
    if args.batch is not None:
        w.B = args.batch
    if args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
