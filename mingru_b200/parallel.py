"""Multi-GPU execution of the scans: batch sharding and sequence parallelism.

The reference is single-device (no collectives anywhere). Two ways to use
several GPUs are provided:

* Batch / head sharding -- every scan is independent across batch rows (and
  heads), so each rank simply runs the ops on its own rows
  (``shard_rows``); there is no collective on the data path.
* Sequence parallelism for very long T (``sp_linear_scan``,
  ``sp_parallel_scan_log``) -- rank r holds time slice r. Each rank
  summarises its slice in one read-only pass (``mgs_*_carry_fwd``: the
  slice's composed forward element per channel), all-gathers the summaries
  (a few (B, D) tensors per rank), composes the earlier slices' summaries
  into the state its slice starts from, and scans its slice from that state
  inside the scan kernels (``mgs_*_fwd_fixup``): inputs read twice, outputs
  written once, no fix-up pass over the outputs. The backward mirrors it:
  each rank summarises its slice's reverse adjoint (``mgs_*_carry_bwd``),
  all-gathers, composes the later slices' summaries into the adjoint entering
  its slice from the right, and runs the backward kernels from it
  (``mgs_*_bwd_fixup``). Every rank runs both all-gathers unconditionally.

Collectives run on the given (default) process group: NCCL between GPUs;
in the CPU tests gloo, with the per-slice operations injected as torch
restatements (``ops``).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .scan_ops import _dense, _dtype_code, _ptr, _require_cuda, _stream, _workspace


def shard_rows(x: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    """Rows ``rank::world``-contiguous block of ``x`` along ``dim`` (batch sharding)."""
    n = x.shape[dim]
    if n % world != 0:
        raise ValueError(f"cannot shard {n} rows over {world} ranks evenly")
    per = n // world
    return x.narrow(dim, rank * per, per)


def _check_same_shape(t: torch.Tensor, group) -> None:
    """Every rank must hold a slice of the same (B, T_local, D) shape."""
    shape = torch.tensor(list(t.shape), dtype=torch.int64, device=t.device)
    world = dist.get_world_size(group)
    shapes = [torch.empty_like(shape) for _ in range(world)]
    dist.all_gather(shapes, shape, group=group)
    if any(not torch.equal(s, shape) for s in shapes):
        raise ValueError(
            "sequence-parallel scan: ranks hold slices of different shapes "
            f"{[tuple(s.tolist()) for s in shapes]}"
        )


def _all_gather(x: torch.Tensor, group) -> torch.Tensor:
    world = dist.get_world_size(group)
    out = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(out, x.contiguous(), group=group)
    return torch.stack(out)


# ------------------------------------------------------------ composition --
# Pure functions of the gathered per-slice summaries G (world, NF, B, D).


def linear_prefix(G: torch.Tensor, rank: int) -> torch.Tensor:
    """(A, B) the slice of `rank` starts from: slices 0 .. rank-1 composed,
    (A1, B1) then (A2, B2) = (A2 A1, A2 B1 + B2)."""
    A = torch.ones_like(G[0, 0])
    Bv = torch.zeros_like(G[0, 1])
    for s in range(rank):
        A, Bv = G[s, 0] * A, G[s, 0] * Bv + G[s, 1]
    return torch.stack([A, Bv])


def linear_suffix(R: torch.Tensor, rank: int) -> torch.Tensor:
    """(Y_A, Y_B) entering the slice of `rank` from the right: the reverse
    summaries (P, Q_A, Q_B) of the later slices applied right to left."""
    ya = torch.zeros_like(R[0, 1])
    yb = torch.zeros_like(R[0, 2])
    for s in range(R.shape[0] - 1, rank, -1):
        ya, yb = R[s, 0] * ya + R[s, 1], R[s, 0] * yb + R[s, 2]
    return torch.stack([ya, yb])


def log_prefix(G: torch.Tensor, rank: int) -> torch.Tensor:
    """Log state the slice of `rank` starts from: slice 0's log h_0 (G[0, 2])
    through the (alpha, nu) summaries of slices 0 .. rank-1."""
    x = G[0, 2]
    for s in range(rank):
        x = torch.logaddexp(x + G[s, 0], G[s, 1])
    return x


def log_suffix(R: torch.Tensor, rank: int) -> torch.Tensor:
    """Adjoint Y entering the slice of `rank` from the right: the reverse
    summaries (P, Q) of the later slices applied right to left."""
    y = torch.zeros_like(R[0, 1])
    for s in range(R.shape[0] - 1, rank, -1):
        y = R[s, 0] * y + R[s, 1]
    return y


# ------------------------------------------------------ per-slice kernels --


class KernelOps:
    """The per-slice operations on this library's kernels (CUDA tensors)."""

    @staticmethod
    def _carry(fn, op, x0, *xs, nf, shape):
        lib = _lib.load()
        Bn, T, D = shape
        with torch.cuda.device(x0.device):
            code = _dtype_code(op, x0)
            agg = torch.empty(nf, Bn, D, dtype=torch.float32, device=x0.device)
            ws = _workspace(lib.mgs_scan_carry_workspace_size(Bn, T, D), x0.device)
            st = fn(*(_ptr(x) for x in (x0,) + xs), _ptr(agg), Bn, T, D, code, _ptr(ws),
                    ws.numel(), _stream(x0))
        _lib.check(st, op)
        return agg

    # linear_scan
    def linear_carry_fwd(self, a, b):
        a, b = _dense(a), _dense(b)
        return self._carry(_lib.load().mgs_linear_scan_carry_fwd, "sp linear carry", a, b, nf=2,
                           shape=a.shape)

    def linear_carry_bwd(self, a, gA, gB):
        a, gA, gB = _dense(a), _dense(gA.to(a.dtype)), _dense(gB.to(a.dtype))
        return self._carry(_lib.load().mgs_linear_scan_carry_bwd, "sp linear carry", a, gA, gB,
                           nf=3, shape=a.shape)

    def linear_fwd_fixup(self, a, b, cin):
        lib = _lib.load()
        a, b, cin = _dense(a), _dense(b), _dense(cin.float())
        Bn, T, D = a.shape
        with torch.cuda.device(a.device):
            code = _dtype_code("sp linear_scan", a)
            A, Bc = torch.empty_like(a), torch.empty_like(b)
            carries = torch.empty(lib.mgs_linear_scan_carry_size(Bn, T, D, code) // 4,
                                  dtype=torch.float32, device=a.device)
            ws = _workspace(lib.mgs_linear_scan_workspace_size(Bn, T, D, code), a.device)
            st = lib.mgs_linear_scan_fwd_fixup(_ptr(a), _ptr(b), _ptr(cin), _ptr(A), _ptr(Bc),
                                               _ptr(carries), Bn, T, D, code, _ptr(ws),
                                               ws.numel(), _stream(a))
        _lib.check(st, "sp linear_scan forward")
        return A, Bc, carries

    def linear_bwd_fixup(self, a, b, carries, yin, gA, gB):
        lib = _lib.load()
        a, b, yin = _dense(a), _dense(b), _dense(yin.float())
        gA, gB = _dense(gA.to(a.dtype)), _dense(gB.to(a.dtype))
        Bn, T, D = a.shape
        with torch.cuda.device(a.device):
            code = _dtype_code("sp linear_scan", a)
            da, db = torch.empty_like(a), torch.empty_like(b)
            ws = _workspace(lib.mgs_linear_scan_workspace_size(Bn, T, D, code), a.device)
            st = lib.mgs_linear_scan_bwd_fixup(_ptr(a), _ptr(b), _ptr(gA), _ptr(gB), _ptr(carries),
                                               _ptr(yin), _ptr(da), _ptr(db), Bn, T, D, code,
                                               _ptr(ws), ws.numel(), _stream(a))
        _lib.check(st, "sp linear_scan backward")
        return da, db

    # parallel_scan_log
    def log_carry_fwd(self, lc, lv):
        lc, lv = _dense(lc), _dense(lv)
        return self._carry(_lib.load().mgs_log_scan_carry_fwd, "sp log carry", lc, lv, nf=2,
                           shape=lc.shape)

    def log_carry_bwd(self, lc, gh):
        lc, gh = _dense(lc), _dense(gh.to(lc.dtype))
        return self._carry(_lib.load().mgs_log_scan_carry_bwd, "sp log carry", lc, gh, nf=2,
                           shape=lc.shape)

    def log_fwd_fixup(self, lc, lv, lh_in):
        lib = _lib.load()
        lc, lv, lh_in = _dense(lc), _dense(lv), _dense(lh_in.float())
        Bn, T, D = lc.shape
        with torch.cuda.device(lc.device):
            code = _dtype_code("sp parallel_scan_log", lc)
            h = torch.empty_like(lc)
            carries = torch.empty(lib.mgs_log_scan_carry_size(Bn, T, D, code) // 4,
                                  dtype=torch.float32, device=lc.device)
            ws = _workspace(lib.mgs_log_scan_workspace_size(Bn, T, D, code), lc.device)
            st = lib.mgs_log_scan_fwd_fixup(_ptr(lc), _ptr(lv), _ptr(lh_in), _ptr(h), _ptr(carries),
                                            Bn, T, D, code, _ptr(ws), ws.numel(), _stream(lc))
        _lib.check(st, "sp parallel_scan_log forward")
        return h, carries

    def log_bwd_fixup(self, lc, lv, lh_in, carries, yin, gh):
        lib = _lib.load()
        lc, lv, lh_in, yin = _dense(lc), _dense(lv), _dense(lh_in.float()), _dense(yin.float())
        gh = _dense(gh.to(lc.dtype))
        Bn, T, D = lc.shape
        with torch.cuda.device(lc.device):
            code = _dtype_code("sp parallel_scan_log", lc)
            dlc, dlv = torch.empty_like(lc), torch.empty_like(lv)
            ws = _workspace(lib.mgs_log_scan_workspace_size(Bn, T, D, code), lc.device)
            st = lib.mgs_log_scan_bwd_fixup(_ptr(lc), _ptr(lv), _ptr(lh_in), _ptr(gh),
                                            _ptr(carries), _ptr(yin), _ptr(dlc), _ptr(dlv), Bn, T,
                                            D, code, _ptr(ws), ws.numel(), _stream(lc))
        _lib.check(st, "sp parallel_scan_log backward")
        return dlc, dlv


# ------------------------------------------------------------ autograd --


class _SPLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, group, ops):
        rank = dist.get_rank(group)
        G = _all_gather(ops.linear_carry_fwd(a, b), group)
        A, Bc, carries = ops.linear_fwd_fixup(a, b, linear_prefix(G, rank))
        ctx.save_for_backward(a, b, carries)
        ctx.group, ctx.ops = group, ops
        ctx.mark_non_differentiable(carries)
        return A, Bc

    @staticmethod
    def backward(ctx, gA, gBc):
        a, b, carries = ctx.saved_tensors
        rank = dist.get_rank(ctx.group)
        gA = torch.zeros_like(a) if gA is None else gA
        gBc = torch.zeros_like(a) if gBc is None else gBc
        R = _all_gather(ctx.ops.linear_carry_bwd(a, gA, gBc), ctx.group)
        da, db = ctx.ops.linear_bwd_fixup(a, b, carries, linear_suffix(R, rank), gA, gBc)
        return da, db, None, None


class _SPLog(torch.autograd.Function):
    @staticmethod
    def forward(ctx, lc, lv, group, ops):
        rank = dist.get_rank(group)
        summary = torch.cat([ops.log_carry_fwd(lc, lv), lv[:, 0].float()[None]])  # (3, B, D)
        G = _all_gather(summary, group)
        lh_in = log_prefix(G, rank)
        h, carries = ops.log_fwd_fixup(lc, lv, lh_in)
        ctx.save_for_backward(lc, lv, lh_in, carries)
        ctx.group, ctx.ops = group, ops
        return h

    @staticmethod
    def backward(ctx, gh):
        lc, lv, lh_in, carries = ctx.saved_tensors
        rank = dist.get_rank(ctx.group)
        gh = torch.zeros_like(lc) if gh is None else gh
        R = _all_gather(ctx.ops.log_carry_bwd(lc, gh), ctx.group)
        dlc, dlv = ctx.ops.log_bwd_fixup(lc, lv, lh_in, carries, log_suffix(R, rank), gh)
        if rank > 0:  # the h_0 slot is read on rank 0 only
            dlv[:, 0] = 0
        return dlc, dlv, None, None


_KERNELS = KernelOps()


def sp_linear_scan(a: torch.Tensor, b: torch.Tensor, group=None, ops=None):
    """Sequence-parallel ``linear_scan`` over the ranks of ``group``.

    ``a``, ``b``: this rank's time slice ``(B, T/world, D)`` (rank order =
    time order, equal slices). Returns this rank's slice of ``(A, Bc)`` of the
    full-length scan, differentiable; every rank must backpropagate through
    its slice (the backward holds one all-gather per rank). ``ops`` (default:
    this library's kernels) supplies the four per-slice operations.
    """
    ops = _KERNELS if ops is None else ops
    if ops is _KERNELS:
        _require_cuda("sp_linear_scan", a, b)
    _check_same_shape(a, group)
    return _SPLinear.apply(a, b, group, ops)


def sp_parallel_scan_log(log_coeffs: torch.Tensor, log_values: torch.Tensor, group=None,
                         ops=None) -> torch.Tensor:
    """Sequence-parallel ``parallel_scan_log`` over the ranks of ``group``.

    ``log_coeffs`` ``(B, T/world, D)``: this rank's time slice;
    ``log_values`` ``(B, T/world + 1, D)``: slot 0 holds log h_0 on rank 0
    (read there only; other ranks' slot 0 is ignored and gets no gradient),
    slots 1.. this rank's log values. Returns this rank's slice of h of the
    full-length scan, differentiable (every rank must backpropagate).
    """
    ops = _KERNELS if ops is None else ops
    if ops is _KERNELS:
        _require_cuda("sp_parallel_scan_log", log_coeffs, log_values)
    _check_same_shape(log_coeffs, group)
    return _SPLog.apply(log_coeffs, log_values, group, ops)
