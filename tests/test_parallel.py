"""Multi-rank host logic on CPU (gloo, world_size 2 and 4): the
sequence-parallel linear and log scans (per-slice carries, all-gather,
prefix / suffix composition, scans from the carried-in state, and the
backward's reverse carries) equal the single-device scans, batch sharding
partitions rows, and failures surface as errors on every rank. The
per-slice operations are the torch restatements of tests/sp_torch_ops.py
(the GPU tests run the kernels)."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sp_torch_ops import TorchOps


def _ref_scan(a, b):
    """Sequential linear scan in torch (the test's host stand-in for the kernel)."""
    A_run = torch.ones_like(a[:, 0])
    B_run = torch.zeros_like(b[:, 0])
    As, Bs = [], []
    for t in range(a.shape[1]):
        A_run = a[:, t] * A_run
        B_run = a[:, t] * B_run + b[:, t]
        As.append(A_run)
        Bs.append(B_run)
    return torch.stack(As, 1), torch.stack(Bs, 1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))


def _sp_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from mingru_b200.parallel import sp_linear_scan

        g = torch.Generator().manual_seed(0)
        B, T, D = 2, 12 * world, 5
        a_full = torch.tanh(torch.randn(B, T, D, generator=g, dtype=torch.float64))
        b_full = torch.randn(B, T, D, generator=g, dtype=torch.float64)
        gA = torch.randn(B, T, D, generator=g, dtype=torch.float64)
        gB = torch.randn(B, T, D, generator=g, dtype=torch.float64)
        per = T // world
        sl = slice(rank * per, (rank + 1) * per)
        a = a_full[:, sl].clone().requires_grad_(True)
        b = b_full[:, sl].clone().requires_grad_(True)
        A, Bc = sp_linear_scan(a, b, ops=TorchOps())
        torch.autograd.backward([A, Bc], [gA[:, sl], gB[:, sl]])
        # single-device reference
        af = a_full.clone().requires_grad_(True)
        bf = b_full.clone().requires_grad_(True)
        Ar, Br = _ref_scan(af, bf)
        torch.autograd.backward([Ar, Br], [gA, gB])
        ok = (torch.allclose(A, Ar[:, sl]) and torch.allclose(Bc, Br[:, sl])
              and torch.allclose(a.grad, af.grad[:, sl]) and torch.allclose(b.grad, bf.grad[:, sl]))
        q.put((rank, ok, None))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported through the queue
        q.put((rank, False, repr(e)))


def _ref_log_scan(lc, lv):
    x = lv[:, 0]
    hs = []
    for t in range(lc.shape[1]):
        x = torch.logaddexp(x + lc[:, t], lv[:, t + 1])
        hs.append(torch.exp(x))
    return torch.stack(hs, 1)


def _sp_log_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from mingru_b200.parallel import sp_parallel_scan_log

        g = torch.Generator().manual_seed(1)
        B, T, D = 2, 10 * world, 4
        k = torch.randn(B, T, D, generator=g, dtype=torch.float64)
        lc_full = -torch.nn.functional.softplus(k)
        lv_full = torch.cat([torch.randn(B, 1, D, generator=g, dtype=torch.float64) * 0.1,
                             -torch.nn.functional.softplus(-k)
                             + torch.randn(B, T, D, generator=g, dtype=torch.float64) * 0.3], 1)
        gh = torch.randn(B, T, D, generator=g, dtype=torch.float64)
        per = T // world
        sl = slice(rank * per, (rank + 1) * per)
        lc = lc_full[:, sl].clone().requires_grad_(True)
        lv_local = lv_full[:, rank * per:(rank + 1) * per + 1].clone()
        if rank > 0:
            lv_local[:, 0] = 123.0  # slot 0 is read on rank 0 only
        lv = lv_local.requires_grad_(True)
        h = sp_parallel_scan_log(lc, lv, ops=TorchOps())
        h.backward(gh[:, sl])
        lcf = lc_full.clone().requires_grad_(True)
        lvf = lv_full.clone().requires_grad_(True)
        hr = _ref_log_scan(lcf, lvf)
        hr.backward(gh)
        want_dlv = lvf.grad[:, rank * per:(rank + 1) * per + 1].clone()
        if rank > 0:
            want_dlv[:, 0] = 0.0
        ok = (torch.allclose(h, hr[:, sl]) and torch.allclose(lc.grad, lcf.grad[:, sl])
              and torch.allclose(lv.grad[:, 1:], want_dlv[:, 1:])
              and torch.allclose(lv.grad[:, 0], want_dlv[:, 0]))
        q.put((rank, ok, None))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported through the queue
        q.put((rank, False, repr(e)))


def _mismatch_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from mingru_b200.parallel import sp_linear_scan

        T = 8 if rank == 0 else 9  # ranks disagree on the slice length
        a = torch.rand(2, T, 3)
        try:
            sp_linear_scan(a, a, ops=TorchOps())
            q.put((rank, False, "no error"))
        except ValueError as e:
            q.put((rank, "different shapes" in str(e), None))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, False, repr(e)))


def _dead_rank_worker(rank, world, port, q):
    """Rank 1 raises before the collective; the others must get an error from
    the bounded process-group timeout, never hang."""
    try:
        _init(rank, world, port)
        from mingru_b200.parallel import sp_linear_scan

        a = torch.rand(2, 6, 3)
        if rank == 1:
            raise RuntimeError("injected failure on rank 1")
        try:
            sp_linear_scan(a, a, ops=TorchOps())
            q.put((rank, False, "collective completed without rank 1"))
        except Exception:  # gloo reports the lost peer / timeout
            q.put((rank, True, None))
    except RuntimeError as e:
        q.put((rank, "injected" in str(e), None))


def _run(fn, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(results)


@pytest.mark.parametrize("world", [2, 4])
def test_sequence_parallel_matches_single_device(world):
    res = _run(_sp_worker, world)
    assert all(ok for _, ok, _ in res), res


@pytest.mark.parametrize("world", [2, 4])
def test_sequence_parallel_log_matches_single_device(world):
    res = _run(_sp_log_worker, world)
    assert all(ok for _, ok, _ in res), res


def test_mismatched_shards_raise_on_every_rank():
    res = _run(_mismatch_worker, 2)
    assert all(ok for _, ok, _ in res), res


def test_lost_rank_is_an_error_not_a_hang():
    res = _run(_dead_rank_worker, 2)
    assert all(ok for _, ok, _ in res), res


def test_shard_rows():
    from mingru_b200.parallel import shard_rows

    x = torch.arange(8 * 3).view(8, 3)
    parts = [shard_rows(x, r, 4) for r in range(4)]
    assert torch.equal(torch.cat(parts), x)
    with pytest.raises(ValueError):
        shard_rows(x, 0, 3)
