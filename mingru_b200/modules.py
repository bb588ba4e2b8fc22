"""Drop-in sequence-mixer modules whose parallel forwards run on the B200 scans.

Same classes, constructor arguments, attribute names, parameter / buffer
names and creation order as the reference package (``mingru`` 0.2.1,
``src/mingru/min_gru.py``), so a reference ``state_dict`` loads unchanged and
a given seed yields the same initial weights:

=================  ==========================  =====================================
class              reference                   scan called by ``forward``
=================  ==========================  =====================================
MinGRU             min_gru.py:1213-1451        ``parallel_scan_log``
SignedMinGRU       min_gru.py:1658-1906        ``linear_scan``
RotationMinGRU     min_gru.py:1909-2362        ``angle_scan_impl`` (k = 2, scale channel)
GivensMinGRU       min_gru.py:2365-2824        ``angle_scan_impl`` (k = block_size)
DeltaMinGRU        min_gru.py:2827-3695        ``delta_scan_impl`` (with decay:
                                               ``delta_gated_scan_impl``)
MinGRUBlock        min_gru.py:3698-3922        (pre-norm residual wrapper)
MinGRUStack        min_gru.py:4019-4336        (stack of blocks)
=================  ==========================  =====================================

The coefficient heads (``nn.Linear`` + elementwise activations) are plain
torch, except MinGRU's without decay, whose softplus / log_g prologue runs
inside the scan kernels (``mingru_gate_scan``). The recurrences run only on
the CUDA kernels (no eager or CPU path: CPU tensors raise ``ValueError``):
``forward`` on the scans above, ``step()`` -- the O(1) per-token recurrence
-- on the fused step kernels of ``step_ops``.
"""

from __future__ import annotations

import math
import warnings
from typing import Literal

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import step_ops
from .scan_ops import (
    angle_scan_impl,
    brickwall_meta,
    delta_gated_scan_impl,
    delta_scan_impl,
    linear_scan,
    mingru_gate_scan,
    parallel_scan_log,
)

Decay = Literal["fixed", "learnable"] | None

# +inf time gaps are capped at this finite value before use (an infinite gap
# would overflow the log-space scan); NaN and negative gaps become 0.
_DELTA_T_POSINF_CAP = 1e10
_DECAY_MIXER_KWARGS = ("decay", "decay_rate", "log1p_delta")


def g(x: torch.Tensor) -> torch.Tensor:
    """Positive activation: ``x + 0.5`` for ``x >= 0``, ``sigmoid(x)`` below."""
    return torch.where(x >= 0, x + 0.5, torch.sigmoid(x))


def log_g(x: torch.Tensor) -> torch.Tensor:
    """``log(g(x))`` with a finite unselected branch (so gradients stay clean)."""
    nonneg = x >= 0
    return torch.where(nonneg, (torch.where(nonneg, x, torch.zeros_like(x)) + 0.5).log(),
                       -F.softplus(-x))


# --------------------------------------------------------------- decay ----


def _match_delta_t_dtype(delta_t, module):
    if delta_t is None:
        return None
    dt = next(module.parameters()).dtype
    return delta_t if delta_t.dtype == dt else delta_t.to(dt)


def _normalize_delta_t(delta_t: torch.Tensor, ndim: int, log1p: bool):
    if delta_t.dim() == ndim + 1:
        if delta_t.size(-1) != 1:
            raise ValueError(
                f"delta_t with {delta_t.dim()} dims must have a trailing size-1 dimension to "
                f"squeeze (got shape {tuple(delta_t.shape)})"
            )
        delta_t = delta_t.squeeze(-1)
    elif delta_t.dim() != ndim:
        raise ValueError(
            f"delta_t must have {ndim} dims (or {ndim + 1} with a trailing size-1 dim to squeeze); "
            f"got shape {tuple(delta_t.shape)}"
        )
    bad = False
    if delta_t.device.type == "cpu":  # inspecting CUDA values would sync the host
        bad = bool(((delta_t < 0) | delta_t.isnan() | delta_t.isinf()).any())
    delta_t = delta_t.nan_to_num(nan=0.0, posinf=_DELTA_T_POSINF_CAP).clamp(min=0)
    return (torch.log1p(delta_t) if log1p else delta_t), bad


def _check_pairing(decay, delta_t) -> None:
    if decay is not None and delta_t is None:
        raise ValueError(f"decay={decay!r} requires delta_t to be provided.")
    if decay is None and delta_t is not None:
        raise ValueError(
            "delta_t was provided but decay is disabled (decay=None); construct the mixer with "
            "decay='fixed' or decay='learnable' to use delta_t."
        )


class DecayMixin:
    """Exponential time decay ``gamma = exp(-lambda * f(delta_t))`` shared by the mixers.

    ``_init_decay`` runs last in each mixer's constructor and draws no random
    numbers, so enabling decay never changes the other weights' init.
    Registers ``decay_rate_buf`` (fixed) or ``rho`` (learnable,
    ``lambda = softplus(rho)``) exactly as the reference does.
    """

    def _init_decay(self, decay, decay_rate, log1p_delta, num_channels):
        if decay not in (None, "fixed", "learnable"):
            raise ValueError(f"decay must be None, 'fixed', or 'learnable' (got {decay!r})")
        if decay is not None and decay_rate <= 0:
            raise ValueError(
                f"decay_rate must be > 0 when decay={decay!r} is enabled (got {decay_rate!r})"
            )
        self.decay = decay
        self.decay_rate = decay_rate
        self.log1p_delta = log1p_delta
        self._warned_negative_dt = False
        if decay == "fixed":
            self.register_buffer("decay_rate_buf", torch.full((), decay_rate))
        elif decay == "learnable":
            self.rho = nn.Parameter(torch.full((num_channels,), math.log(math.expm1(decay_rate))))

    def _decay_lambda(self):
        return self.decay_rate_buf if self.decay == "fixed" else F.softplus(self.rho)

    def _decay_gamma(self, dt):
        return torch.exp(-self._decay_lambda() * dt.unsqueeze(-1))

    def _prepare_decay(self, delta_t, canonical_ndim):
        _check_pairing(self.decay, delta_t)
        if delta_t is None:
            return None
        dt, bad = _normalize_delta_t(delta_t, canonical_ndim, self.log1p_delta)
        if bad and not self._warned_negative_dt:
            warnings.warn(
                "delta_t contains negative, NaN, or infinite entries; sanitizing to finite, "
                "non-negative values.",
                stacklevel=3,
            )
            self._warned_negative_dt = True
        return dt


# -------------------------------------------------------------- mixers ----


class MinGRU(DecayMixin, nn.Module):
    """minGRU (Feng et al. 2024) in log space: ``h_t = (1 - z_t) h_{t-1} + z_t g(h~_t)``.

    ``forward(x (B, T, input_size), h_0 (B, 1, hidden)=None, delta_t=None)``
    returns all states ``(B, T, hidden)`` through ``parallel_scan_log``.
    """

    def __init__(self, input_size, hidden_size, bias=True, learnable_h0=False, decay: Decay = None,
                 decay_rate=1.0, log1p_delta=False):
        super().__init__()
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.linear_z = nn.Linear(input_size, hidden_size, bias=bias)
        self.linear_h = nn.Linear(input_size, hidden_size, bias=bias)
        self.h0_pre = nn.Parameter(torch.zeros(1, 1, hidden_size)) if learnable_h0 else None
        self._init_decay(decay, decay_rate, log1p_delta, hidden_size)

    def forward(self, x, h_0=None, delta_t=None):
        B = x.size(0)
        if h_0 is None:
            if self.h0_pre is not None:
                log_h0 = log_g(self.h0_pre).expand(B, 1, self.hidden_size)
            else:
                log_h0 = torch.full((B, 1, self.hidden_size), math.log(0.5), dtype=x.dtype,
                                    device=x.device)
        else:
            torch._assert_async((h_0 >= 0).all(), "h_0 must be a non-negative real hidden state "
                                "(an output of forward()/step()), not a pre-activation.")
            log_h0 = h_0.clamp_min(torch.finfo(h_0.dtype).tiny).log()
        k = self.linear_z(x)
        dt = self._prepare_decay(delta_t, canonical_ndim=2)
        if dt is None:  # the coefficient prologue runs inside the scan kernels
            return mingru_gate_scan(k, self.linear_h(x), log_h0.to(k.dtype))
        log_z = -F.softplus(-k)
        log_coeffs = -F.softplus(k) - self._decay_lambda() * dt.unsqueeze(-1)
        log_values = torch.cat([log_h0.to(log_z.dtype), log_z + log_g(self.linear_h(x))], dim=1)
        return parallel_scan_log(log_coeffs, log_values)

    @torch.no_grad()
    def step(self, x_t, h_prev=None, delta_t=None):
        if h_prev is None:
            h_prev = (g(self.h0_pre)[:, 0].expand(x_t.size(0), self.hidden_size)
                      if self.h0_pre is not None
                      else x_t.new_full((x_t.size(0), self.hidden_size), 0.5))
        dt = self._prepare_decay(delta_t, canonical_ndim=1)
        gamma = self._decay_gamma(dt).to(x_t.dtype) if dt is not None else None
        return step_ops.mingru_step(self.linear_z(x_t), self.linear_h(x_t), h_prev.to(x_t.dtype),
                                    None if gamma is None else gamma.expand(h_prev.shape))

    def extra_repr(self):
        return f"input_size={self.input_size}, hidden_size={self.hidden_size}"


class SignedMinGRU(DecayMixin, nn.Module):
    """minGRU with signed diagonal transitions ``a_t = tanh(s_t)`` (linear-space scan)."""

    def __init__(self, input_size, hidden_size, bias=True, learnable_h0=False, coupled=False,
                 decay: Decay = None, decay_rate=1.0, log1p_delta=False):
        super().__init__()
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.coupled = coupled
        self.linear_z = nn.Linear(input_size, hidden_size, bias=bias)
        self.linear_h = nn.Linear(input_size, hidden_size, bias=bias)
        self.linear_s = nn.Linear(input_size, hidden_size, bias=bias)
        self.h0 = nn.Parameter(torch.zeros(1, 1, hidden_size)) if learnable_h0 else None
        self._init_decay(decay, decay_rate, log1p_delta, hidden_size)

    def _coeffs(self, x, dt=None):
        z = torch.sigmoid(self.linear_z(x))
        s = torch.tanh(self.linear_s(x))
        a = (1 - z) * s if self.coupled else s
        if dt is not None:
            a = self._decay_gamma(dt) * a
        return a, z * self.linear_h(x)

    def forward(self, x, h_0=None, delta_t=None):
        if h_0 is None:
            h_0 = (self.h0.expand(x.size(0), 1, self.hidden_size) if self.h0 is not None
                   else x.new_zeros(x.size(0), 1, self.hidden_size))
        a, b = self._coeffs(x, self._prepare_decay(delta_t, canonical_ndim=2))
        A, Bc = linear_scan(a, b)
        return A * h_0 + Bc

    @torch.no_grad()
    def step(self, x_t, h_prev=None, delta_t=None):
        if h_prev is None:
            h_prev = (self.h0[:, 0].expand(x_t.size(0), self.hidden_size) if self.h0 is not None
                      else x_t.new_zeros(x_t.size(0), self.hidden_size))
        dt = self._prepare_decay(delta_t, canonical_ndim=1)
        gamma = self._decay_gamma(dt).to(x_t.dtype).expand(h_prev.shape) if dt is not None else None
        return step_ops.signed_step(self.linear_z(x_t), self.linear_s(x_t), self.linear_h(x_t),
                                    h_prev.to(x_t.dtype), gamma, self.coupled)

    def extra_repr(self):
        return f"input_size={self.input_size}, hidden_size={self.hidden_size}, coupled={self.coupled}"


class RotationMinGRU(DecayMixin, nn.Module):
    """2x2 block-rotation minGRU: ``h_t = gamma R(theta_t) diag(1, tanh u_t) h_{t-1} + b_t``
    per planar block; the recurrence runs on the angle-fused kernel (k = 2)."""

    def __init__(self, input_size, hidden_size, bias=True, snap=(2, 3, 4, 6), decay: Decay = None,
                 decay_rate=1.0, log1p_delta=False):
        super().__init__()
        if hidden_size % 2 != 0:
            raise ValueError(
                f"RotationMinGRU requires an even hidden_size (got {hidden_size}); state is "
                "n = hidden_size / 2 planar 2D blocks."
            )
        if snap is not None and (len(snap) == 0 or any(k < 1 for k in snap)):
            raise ValueError(f"snap must be None or a non-empty tuple of positive ints (got {snap!r})")
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.n_blocks = hidden_size // 2
        self.snap = snap
        self.linear_z = nn.Linear(input_size, hidden_size, bias=bias)
        self.linear_h = nn.Linear(input_size, hidden_size, bias=bias)
        self.linear_theta = nn.Linear(input_size, self.n_blocks, bias=bias)
        self.linear_u = nn.Linear(input_size, self.n_blocks, bias=bias)
        self.h0 = nn.Parameter(torch.randn(1, 1, hidden_size) * 0.5)
        if snap is not None:
            self.register_buffer(
                "snap_step",
                torch.tensor([2 * math.pi / snap[j % len(snap)] for j in range(self.n_blocks)]),
            )
        self._init_decay(decay, decay_rate, log1p_delta, self.n_blocks)

    def _theta(self, x):
        theta = self.linear_theta(x)
        if self.snap is not None:  # straight-through snap to a multiple of 2*pi/snap_j
            snapped = torch.round(theta / self.snap_step) * self.snap_step
            theta = theta + (snapped - theta).detach()
        return theta

    def _meta(self, device):
        cache = getattr(self, "_angle_meta_cache", None)
        if cache is None or cache[0].device != device:
            cache = brickwall_meta(1, 2, device)
            self._angle_meta_cache = cache
        return cache

    def forward(self, x, h_0=None, delta_t=None):
        B, T, _ = x.shape
        n = self.n_blocks
        if h_0 is None:
            h_0 = self.h0.expand(B, 1, self.hidden_size)
        dt = self._prepare_decay(delta_t, canonical_ndim=2)
        theta = self._theta(x).view(B, T, n, 1, 1)
        scale = torch.tanh(self.linear_u(x))
        b = (torch.sigmoid(self.linear_z(x)) * self.linear_h(x)).reshape(B, T, n, 2)
        gamma = (self._decay_gamma(dt).expand(B, T, n) if dt is not None
                 else torch.ones(B, T, n, dtype=x.dtype, device=x.device))
        h = angle_scan_impl(theta, scale, gamma, b, h_0.reshape(B, n, 2).to(b.dtype), *self._meta(x.device),
                            has_scale=1, has_decay=int(dt is not None))
        return h.reshape(B, T, self.hidden_size)

    @torch.no_grad()
    def step(self, x_t, h_prev=None, delta_t=None):
        B = x_t.size(0)
        if h_prev is None:
            h_prev = self.h0.expand(B, 1, self.hidden_size)[:, 0]
        dt = self._prepare_decay(delta_t, canonical_ndim=1)
        gamma = (self._decay_gamma(dt).to(x_t.dtype).expand(B, self.n_blocks) if dt is not None
                 else None)
        return step_ops.rotation_step(self._theta(x_t), self.linear_u(x_t), self.linear_z(x_t),
                                      self.linear_h(x_t), h_prev.to(x_t.dtype), gamma)

    def extra_repr(self):
        return f"input_size={self.input_size}, hidden_size={self.hidden_size}, snap={self.snap}"


class GivensMinGRU(DecayMixin, nn.Module):
    """k x k block-orthogonal minGRU: each block's transition is ``gamma`` times
    ``rounds`` brick-wall rounds of Givens rotations; the recurrence runs on the
    angle-fused kernel (the k x k matrices are never built)."""

    def __init__(self, input_size, hidden_size, bias=True, block_size=8, rounds=3,
                 decay: Decay = None, decay_rate=1.0, log1p_delta=False):
        super().__init__()
        if block_size % 2 != 0:
            raise ValueError(
                f"GivensMinGRU requires an even block_size (got {block_size}); brick-wall Givens "
                "rounds pair the k state dims into k/2 disjoint planes."
            )
        if hidden_size % block_size != 0:
            raise ValueError(
                f"GivensMinGRU requires hidden_size ({hidden_size}) divisible by block_size "
                f"({block_size}); state is n_blocks = hidden_size / block_size blocks of "
                "block_size dims."
            )
        if rounds < 1:
            raise ValueError(f"GivensMinGRU requires rounds >= 1 (got {rounds})")
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.k = block_size
        self.n_blocks = hidden_size // block_size
        self.rounds = rounds
        half = block_size // 2
        self.linear_theta = nn.Linear(input_size, self.n_blocks * rounds * half, bias=bias)
        self.linear_z = nn.Linear(input_size, hidden_size, bias=bias)
        self.linear_h = nn.Linear(input_size, hidden_size, bias=bias)
        self.h0 = nn.Parameter(torch.randn(1, 1, hidden_size) * 0.5)
        for r in range(rounds):  # plane index buffers of round r: (i, i+1 mod k), i = r%2 + 2m
            first = torch.arange(r % 2, block_size, 2) % block_size
            self.register_buffer(f"_pi{r}", first)
            self.register_buffer(f"_pj{r}", (first + 1) % block_size)
        self._init_decay(decay, decay_rate, log1p_delta, self.n_blocks)

    def _meta(self, device):
        cache = getattr(self, "_angle_meta_cache", None)
        if cache is None or cache[0].device != device:
            cache = brickwall_meta(self.rounds, self.k, device)
            self._angle_meta_cache = cache
        return cache

    def forward(self, x, h_0=None, delta_t=None):
        B, T, _ = x.shape
        n, k, R = self.n_blocks, self.k, self.rounds
        if h_0 is None:
            h_0 = self.h0.expand(B, 1, self.hidden_size)
        dt = self._prepare_decay(delta_t, canonical_ndim=2)
        theta = self.linear_theta(x).view(B, T, n, R, k // 2)
        b = (torch.sigmoid(self.linear_z(x)) * self.linear_h(x)).reshape(B, T, n, k)
        gamma = (self._decay_gamma(dt).expand(B, T, n) if dt is not None
                 else torch.ones(B, T, n, dtype=x.dtype, device=x.device))
        scale = torch.ones(B, T, n, dtype=x.dtype, device=x.device)
        h = angle_scan_impl(theta, scale, gamma, b, h_0.reshape(B, n, k).to(b.dtype), *self._meta(x.device),
                            has_scale=0, has_decay=int(dt is not None))
        return h.reshape(B, T, self.hidden_size)

    @torch.no_grad()
    def step(self, x_t, h_prev=None, delta_t=None):
        B = x_t.size(0)
        n, k, R = self.n_blocks, self.k, self.rounds
        if h_prev is None:
            h_prev = self.h0.expand(B, 1, self.hidden_size)[:, 0]
        dt = self._prepare_decay(delta_t, canonical_ndim=1)
        gamma = self._decay_gamma(dt).to(x_t.dtype).expand(B, n) if dt is not None else None
        theta = self.linear_theta(x_t).view(B, n, R, k // 2)
        return step_ops.givens_step(theta, self.linear_z(x_t), self.linear_h(x_t),
                                    h_prev.to(x_t.dtype), gamma)

    def extra_repr(self):
        return (f"input_size={self.input_size}, hidden_size={self.hidden_size}, "
                f"block_size={self.k}, rounds={self.rounds}")


class DeltaMinGRU(DecayMixin, nn.Module):
    """Delta-rule mixer (DeltaNet / DeltaProduct): per head a d_k x d_v memory
    ``H`` updated by ``nh`` rank-1 corrections per token, read by ``q``; the
    parallel forward is the chunked-WY kernel ``delta_scan_impl``."""

    carries_matrix_state: bool = True

    def __init__(self, input_size, hidden_size, bias=True, n_heads=4, nh=1, d_k=None, d_v=None,
                 chunk_size=64, decay: Decay = None, decay_rate=1.0, log1p_delta=False):
        super().__init__()
        if n_heads <= 0:
            raise ValueError(f"n_heads must be positive (got {n_heads})")
        if nh <= 0:
            raise ValueError(f"nh must be positive (got {nh})")
        if chunk_size <= 0:
            raise ValueError(f"chunk_size must be positive (got {chunk_size})")
        if d_k is None and hidden_size % n_heads != 0:
            raise ValueError(
                f"hidden_size ({hidden_size}) must be divisible by n_heads ({n_heads}) when d_k is "
                "not given explicitly"
            )
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.n_heads = n_heads
        self.nh = nh
        self.d_k = d_k if d_k is not None else hidden_size // n_heads
        self.d_v = d_v if d_v is not None else self.d_k
        self.chunk_size = chunk_size
        self.linear_q = nn.Linear(input_size, n_heads * self.d_k, bias=bias)
        self.linear_k = nn.ModuleList(
            nn.Linear(input_size, n_heads * self.d_k, bias=bias) for _ in range(nh))
        self.linear_v = nn.ModuleList(
            nn.Linear(input_size, n_heads * self.d_v, bias=bias) for _ in range(nh))
        self.linear_beta = nn.ModuleList(nn.Linear(input_size, n_heads, bias=bias) for _ in range(nh))
        self.out_proj = nn.Linear(n_heads * self.d_v, hidden_size, bias=bias)
        self._warned_fp32_decay_saturation = False
        self._init_decay(decay, decay_rate, log1p_delta, num_channels=self.n_heads)

    def _coeffs(self, x):
        lead = x.shape[:-1]
        q = self.linear_q(x).view(*lead, self.n_heads, self.d_k)
        ks = [F.normalize(lin(x).view(*lead, self.n_heads, self.d_k), dim=-1) for lin in self.linear_k]
        vs = [lin(x).view(*lead, self.n_heads, self.d_v) for lin in self.linear_v]
        betas = [2 * torch.sigmoid(lin(x)) for lin in self.linear_beta]
        return q, ks, vs, betas

    def forward(self, x, h_0=None, delta_t=None, return_state=False):
        delta_t = _match_delta_t_dtype(delta_t, self)
        dt = self._prepare_decay(delta_t, canonical_ndim=2)
        B, T, _ = x.shape
        expected = (B, 1, self.n_heads * self.d_k * self.d_v)
        if h_0 is None:
            H = x.new_zeros(B, self.n_heads, self.d_k, self.d_v)
        else:
            if tuple(h_0.shape) != expected:
                raise ValueError(f"h_0 must have shape {expected} (got {tuple(h_0.shape)})")
            H = h_0.reshape(B, self.n_heads, self.d_k, self.d_v)
        if T == 0:
            y = x.new_zeros(B, 0, self.n_heads * self.d_v)
            H = H.clone()
        else:
            q, ks, vs, betas = self._coeffs(x)
            K = torch.stack(ks, dim=2).permute(0, 3, 1, 2, 4)
            V = torch.stack(vs, dim=2).permute(0, 3, 1, 2, 4)
            beta = torch.stack(betas, dim=2).permute(0, 3, 1, 2)
            Q = q.permute(0, 2, 1, 3)
            if dt is None:
                y, H_T = delta_scan_impl(Q, K, V, beta, H.to(torch.float32),
                                         chunk_size=self.chunk_size)
            else:  # per-token log decay -lambda dt per head (min_gru.py:3379-3386)
                lam = self._decay_lambda()
                log_gamma = -lam.reshape(1, -1, 1) * dt.unsqueeze(1)
                y, H_T = delta_gated_scan_impl(Q, K, V, beta, H.to(torch.float32),
                                               log_gamma.expand(B, self.n_heads, T),
                                               chunk_size=self.chunk_size)
            H = H_T.to(x.dtype)
            y = y.permute(0, 2, 1, 3).reshape(B, T, self.n_heads * self.d_v).to(x.dtype)
        y = self.out_proj(y)
        if return_state:
            return y, H.reshape(*expected)
        return y

    @torch.no_grad()
    def step(self, x_t, h_prev=None, delta_t=None):
        delta_t = _match_delta_t_dtype(delta_t, self)
        dt = self._prepare_decay(delta_t, canonical_ndim=1)
        B = x_t.size(0)
        expected = (B, self.n_heads * self.d_k * self.d_v)
        if h_prev is None:
            H = x_t.new_zeros(B, self.n_heads, self.d_k, self.d_v)
        else:
            if tuple(h_prev.shape) != expected:
                raise ValueError(f"h_prev must have shape {expected} (got {tuple(h_prev.shape)})")
            H = h_prev.reshape(B, self.n_heads, self.d_k, self.d_v)
        gamma = (self._decay_gamma(dt).to(x_t.dtype).expand(B, self.n_heads) if dt is not None
                 else None)
        q, ks, vs, betas = self._coeffs(x_t)
        y, H = step_ops.delta_step(q, torch.stack(ks, 2), torch.stack(vs, 2), torch.stack(betas, 2),
                                   H.to(x_t.dtype), gamma)
        return self.out_proj(y.reshape(B, self.n_heads * self.d_v)), H.reshape(*expected)

    def extra_repr(self):
        return (f"input_size={self.input_size}, hidden_size={self.hidden_size}, "
                f"n_heads={self.n_heads}, nh={self.nh}, d_k={self.d_k}, d_v={self.d_v}, "
                f"chunk_size={self.chunk_size}")


# ------------------------------------------------------ block / stack -----


class MinGRUBlock(nn.Module):
    """Pre-norm residual block: ``x + mixer(LN(x))`` then ``x + MLP(LN(x))``."""

    _MIXER_CLASSES: dict[str, tuple[type[nn.Module], bool]] = {
        "log": (MinGRU, True),
        "signed": (SignedMinGRU, True),
        "rotation": (RotationMinGRU, False),
        "givens": (GivensMinGRU, False),
        "delta": (DeltaMinGRU, False),
    }

    def __init__(self, d_model, mlp_expansion=4, dropout=0.0, learnable_h0=False, mixer="log",
                 mixer_kwargs=None):
        super().__init__()
        if mixer not in self._MIXER_CLASSES:
            raise ValueError(f"unknown mixer {mixer!r}; expected one of {sorted(self._MIXER_CLASSES)}")
        kwargs = dict(mixer_kwargs) if mixer_kwargs else {}
        self.norm1 = nn.LayerNorm(d_model)
        cls, takes_h0 = self._MIXER_CLASSES[mixer]
        if takes_h0:
            kwargs["learnable_h0"] = learnable_h0
        self.mingru = cls(d_model, d_model, **kwargs)
        self.drop = nn.Dropout(dropout)
        if mlp_expansion > 0:
            self.norm2 = nn.LayerNorm(d_model)
            self.mlp = nn.Sequential(
                nn.Linear(d_model, mlp_expansion * d_model),
                nn.GELU(),
                nn.Dropout(dropout),
                nn.Linear(mlp_expansion * d_model, d_model),
            )
        else:
            self.norm2 = None
            self.mlp = None

    def forward(self, x, h_0=None, delta_t=None):
        delta_t = _match_delta_t_dtype(delta_t, self.mingru)
        if getattr(self.mingru, "carries_matrix_state", False):
            h_seq, state = self.mingru(self.norm1(x), h_0, delta_t, return_state=True)
        else:
            h_seq = self.mingru(self.norm1(x), h_0, delta_t)
            state = h_seq[:, -1:]
        x = x + self.drop(h_seq)
        if self.mlp is not None:
            x = x + self.mlp(self.norm2(x))
        return x, state

    @torch.no_grad()
    def step(self, x_t, h_prev, delta_t=None):
        delta_t = _match_delta_t_dtype(delta_t, self.mingru)
        if getattr(self.mingru, "carries_matrix_state", False):
            y_t, state = self.mingru.step(self.norm1(x_t), h_prev, delta_t)
        else:
            y_t = self.mingru.step(self.norm1(x_t), h_prev, delta_t)
            state = y_t
        x_t = x_t + y_t
        if self.mlp is not None:
            x_t = x_t + self.mlp(self.norm2(x_t))
        return x_t, state


def _resolve_stack_mixer_spec(mixer, mixer_kwargs, n_layers):
    """Per-layer mixer names and per-type kwargs (the reference's
    ``_resolve_stack_mixer_spec`` contract, min_gru.py:3925-4016)."""
    valid = MinGRUBlock._MIXER_CLASSES
    if isinstance(mixer, str):
        if mixer_kwargs:
            hits = sorted(k for k in mixer_kwargs if k in valid)
            if hits:
                raise ValueError(
                    f"mixer={mixer!r} is a single mixer name, so mixer_kwargs must be a flat dict "
                    f"of that mixer's constructor kwargs; got key(s) matching a mixer type name "
                    f"instead ({hits!r}), which is the schema for a list mixer."
                )
        return [mixer] * n_layers, {mixer: mixer_kwargs}
    if isinstance(mixer, list):
        if len(mixer) != n_layers:
            raise ValueError(f"mixer list length ({len(mixer)}) must equal n_layers ({n_layers})")
        unknown = sorted({m for m in mixer if m not in valid})
        if unknown:
            raise ValueError(
                f"unknown mixer name(s) {unknown!r} in mixer list; expected one of {sorted(valid)}"
            )
        present = set(mixer)
        if mixer_kwargs is None:
            return list(mixer), {m: None for m in present}
        bad = sorted(k for k in mixer_kwargs if k not in valid or k not in present)
        if bad:
            raise ValueError(
                f"mixer_kwargs keys must name a mixer type present in mixer={mixer!r} (one of "
                f"{sorted(present)}); got unexpected key(s) {bad!r}."
            )
        return list(mixer), {m: mixer_kwargs.get(m) for m in present}
    raise ValueError(f"mixer must be a str or list[str] (got {type(mixer).__name__})")


class MinGRUStack(nn.Module):
    """``in_proj`` -> ``n_layers`` MinGRUBlocks -> LayerNorm, with per-block state."""

    def __init__(self, input_size, d_model, n_layers, mlp_expansion=4, dropout=0.0,
                 learnable_h0=False, mixer="log", mixer_kwargs=None, decay_layers="all"):
        super().__init__()
        if decay_layers not in ("all", "last"):
            raise ValueError(f"decay_layers must be 'all' or 'last' (got {decay_layers!r})")
        self.decay_layers = decay_layers
        self.in_proj = nn.Linear(input_size, d_model) if input_size != d_model else nn.Identity()
        names, by_type = _resolve_stack_mixer_spec(mixer, mixer_kwargs, n_layers)
        no_decay = {
            m: ({k: v for k, v in kw.items() if k not in _DECAY_MIXER_KWARGS}
                if decay_layers == "last" and kw else kw)
            for m, kw in by_type.items()
        }
        if names.count("rotation") > 1:
            warnings.warn(
                f"stack contains more than one 'rotation' block ({names.count('rotation')} of "
                f"{n_layers}): the straight-through snap discontinuity can compound across "
                "rotation layers; proceeding anyway.",
                stacklevel=2,
            )
        self.blocks = nn.ModuleList(
            MinGRUBlock(d_model, mlp_expansion, dropout, learnable_h0, name,
                        by_type[name] if i == n_layers - 1 else no_decay[name])
            for i, name in enumerate(names)
        )
        self.norm_out = nn.LayerNorm(d_model)

    def _check_delta_t_has_decay(self, delta_t):
        if not any(blk.mingru.decay is not None for blk in self.blocks):
            _check_pairing(None, delta_t)

    def init_state(self):
        return [None] * len(self.blocks)

    def forward(self, x, state=None, delta_t=None):
        if state is None:
            state = self.init_state()
        self._check_delta_t_has_decay(delta_t)
        x = self.in_proj(x)
        new_state = []
        for blk, h0 in zip(self.blocks, state):
            x, h_last = blk(x, h0, delta_t if blk.mingru.decay is not None else None)
            new_state.append(h_last)
        return self.norm_out(x), new_state

    @torch.no_grad()
    def step(self, x_t, state, delta_t=None):
        self._check_delta_t_has_decay(delta_t)
        x_t = self.in_proj(x_t)
        new_state = []
        for blk, h_prev in zip(self.blocks, state):
            x_t, h = blk.step(x_t, h_prev, delta_t if blk.mingru.decay is not None else None)
            new_state.append(h)
        return self.norm_out(x_t), new_state
