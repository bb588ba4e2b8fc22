"""Multi-GPU execution of the scans: batch sharding and sequence parallelism.

The reference is single-device (no collectives anywhere). Two ways to use
several GPUs are provided:

* Batch / head sharding -- every scan is independent across batch rows (and
  heads), so each rank simply runs the ops on its own rows
  (``shard_rows``); there is no collective on the data path.
* Sequence parallelism for very long T (``sp_linear_scan``) -- rank r holds
  time slice r of ``a`` and ``b``. It scans its slice locally from the
  identity, all-gathers only each shard's end element (the composed
  transition ``prod a`` and the end state, two (B, D) tensors per rank),
  composes the prefix of the earlier shards on every rank, and fixes its
  slice up: ``A_t <- A_t * A_in``, ``Bc_t <- A_t * Bc_in + Bc_t``. The
  backward differentiates through the same steps; the all-gather's adjoint
  is an all-reduce of the gathered gradients, so every rank receives the
  gradient flowing into its end element from all later shards.

Collectives run on the default process group (NCCL between GPUs; gloo in
the CPU tests, where a host scan function is injected).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .scan_ops import linear_scan


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


def _compose_prefix(ends_A, ends_B, upto: int):
    """Composition of shards 0 .. upto-1: (A1, B1) then (A2, B2) = (A2 A1, A2 B1 + B2)."""
    A_in = torch.ones_like(ends_A[0])
    B_in = torch.zeros_like(ends_B[0])
    for j in range(upto):
        A_in, B_in = ends_A[j] * A_in, ends_A[j] * B_in + ends_B[j]
    return A_in, B_in


class _SPFixup(torch.autograd.Function):
    """Carry exchange + fix-up of a sequence-parallel linear scan.

    Forward: all-gather every shard's end element, compose the shards before
    this rank, apply the carry to the local outputs. Backward: gradients of the
    local outputs, plus the gradient of this rank's carry pushed back to the
    end elements of every earlier shard; one all-reduce (run by every rank,
    always) delivers each shard the sum of what later shards send it.
    """

    @staticmethod
    def forward(ctx, A_loc, B_loc, group):
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        ends = torch.stack([A_loc[:, -1], B_loc[:, -1]]).contiguous()  # (2, B, D)
        gathered = [torch.empty_like(ends) for _ in range(world)]
        dist.all_gather(gathered, ends, group=group)
        gathered = torch.stack(gathered)  # (world, 2, B, D)
        A_in, B_in = _compose_prefix(gathered[:, 0], gathered[:, 1], rank)
        ctx.save_for_backward(A_loc, gathered, A_in, B_in)
        ctx.group = group
        return A_loc * A_in.unsqueeze(1), A_loc * B_in.unsqueeze(1) + B_loc

    @staticmethod
    def backward(ctx, gA, gBc):
        A_loc, gathered, A_in, B_in = ctx.saved_tensors
        group = ctx.group
        rank = dist.get_rank(group)
        gA = torch.zeros_like(A_loc) if gA is None else gA
        gBc = torch.zeros_like(A_loc) if gBc is None else gBc
        gA_loc = gA * A_in.unsqueeze(1) + gBc * B_in.unsqueeze(1)
        gB_loc = gBc.clone()
        gA_in = (gA * A_loc).sum(1)
        gB_in = (gBc * A_loc).sum(1)
        with torch.enable_grad():
            ends = gathered.detach().requires_grad_(True)
            A_c, B_c = _compose_prefix(ends[:, 0], ends[:, 1], rank)
            if rank > 0:
                (g_ends,) = torch.autograd.grad((A_c, B_c), (ends,), (gA_in, gB_in))
            else:
                g_ends = torch.zeros_like(ends)
        dist.all_reduce(g_ends, op=dist.ReduceOp.SUM, group=group)
        gA_loc[:, -1] += g_ends[rank, 0]
        gB_loc[:, -1] += g_ends[rank, 1]
        return gA_loc, gB_loc, None


def sp_linear_scan(a: torch.Tensor, b: torch.Tensor, group=None, scan_fn=linear_scan):
    """Sequence-parallel ``linear_scan`` over the ranks of ``group``.

    ``a``, ``b``: this rank's time slice ``(B, T/world, D)`` (rank order =
    time order, equal slices). Returns this rank's slice of ``(A, Bc)`` of the
    full-length scan, differentiable; every rank must backpropagate through
    its slice (the backward holds one all-reduce per rank). ``scan_fn`` is
    the local scan (the CUDA kernel by default).
    """
    _check_same_shape(a, group)
    A_loc, B_loc = scan_fn(a, b)
    return _SPFixup.apply(A_loc, B_loc, group)
