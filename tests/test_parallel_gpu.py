"""Sequence-parallel linear_scan and parallel_scan_log with the CUDA kernels
over NCCL (needs >= 2 GPUs; skipped otherwise): every rank's slice of the
forward outputs and of the input gradients equals the single-GPU
full-length scan."""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        import mingru_b200 as mb
        from mingru_b200.parallel import sp_linear_scan, sp_parallel_scan_log

        g = torch.Generator().manual_seed(0)
        B, T, D = 4, 512 * world, 256
        a = torch.tanh(torch.randn(B, T, D, generator=g)).to(dev)
        b = torch.randn(B, T, D, generator=g).to(dev)
        gA = torch.randn(B, T, D, generator=g).to(dev)
        gB = torch.randn(B, T, D, generator=g).to(dev)
        per = T // world
        sl = slice(rank * per, (rank + 1) * per)
        al = a[:, sl].clone().requires_grad_(True)
        bl = b[:, sl].clone().requires_grad_(True)
        A, Bc = sp_linear_scan(al, bl)
        torch.autograd.backward([A, Bc], [gA[:, sl], gB[:, sl]])
        af, bf = a.clone().requires_grad_(True), b.clone().requires_grad_(True)
        Ar, Br = mb.linear_scan(af, bf)
        torch.autograd.backward([Ar, Br], [gA, gB])
        tol = dict(rtol=1e-5, atol=1e-5)
        ok = (torch.allclose(A, Ar[:, sl], **tol) and torch.allclose(Bc, Br[:, sl], **tol)
              and torch.allclose(al.grad, af.grad[:, sl], rtol=1e-4, atol=1e-4)
              and torch.allclose(bl.grad, bf.grad[:, sl], rtol=1e-4, atol=1e-4))
        # parallel_scan_log: log h_0 in slot 0 of rank 0's log values
        k = torch.randn(B, T, D, generator=g).to(dev)
        lc = -torch.nn.functional.softplus(k)
        lv = torch.cat([torch.full((B, 1, D), -0.7, device=dev),
                        -torch.nn.functional.softplus(-k) + 0.3 * torch.randn(B, T, D, generator=g).to(dev)], 1)
        gh = torch.randn(B, T, D, generator=g).to(dev)
        lcl = lc[:, sl].clone().requires_grad_(True)
        lvl = lv[:, sl.start:sl.stop + 1].clone().requires_grad_(True)
        h = sp_parallel_scan_log(lcl, lvl)
        h.backward(gh[:, sl])
        lcf, lvf = lc.clone().requires_grad_(True), lv.clone().requires_grad_(True)
        hr = mb.parallel_scan_log(lcf, lvf)
        hr.backward(gh)
        ok = ok and (torch.allclose(h, hr[:, sl], **tol)
                     and torch.allclose(lcl.grad, lcf.grad[:, sl], rtol=1e-4, atol=1e-4)
                     and torch.allclose(lvl.grad[:, 1:], lvf.grad[:, sl.start + 1:sl.stop + 1],
                                        rtol=1e-4, atol=1e-4))
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()
        q.put((rank, ok, None))
    except Exception as e:  # pragma: no cover
        q.put((rank, False, repr(e)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs >= 2 GPUs")
def test_sequence_parallel_nccl():
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert all(ok for _, ok, _ in res), res
