"""Torch restatements of the four per-slice sequence-parallel operations, for
the multi-rank CPU tests (gloo). TEST INFRASTRUCTURE: the GPU path runs the
kernels (mingru_b200.parallel.KernelOps); these follow the same recurrences
one step at a time, so the host-side composition and collectives can be
tested without a GPU."""

from __future__ import annotations

import torch


class TorchOps:
    # ---- linear_scan: h_t = a_t h_{t-1} + b_t
    def linear_carry_fwd(self, a, b):
        A = torch.ones_like(a[:, 0])
        Bv = torch.zeros_like(b[:, 0])
        for t in range(a.shape[1]):
            Bv = a[:, t] * Bv + b[:, t]
            A = a[:, t] * A
        return torch.stack([A, Bv])

    def linear_fwd_fixup(self, a, b, cin):
        A, Bv = cin[0].to(a.dtype), cin[1].to(a.dtype)
        As, Bs = [], []
        for t in range(a.shape[1]):
            A = a[:, t] * A
            Bv = a[:, t] * Bv + b[:, t]
            As.append(A)
            Bs.append(Bv)
        return torch.stack(As, 1), torch.stack(Bs, 1), cin.clone()

    def linear_carry_bwd(self, a, gA, gB):
        P = torch.ones_like(a[:, 0])
        qa = torch.zeros_like(a[:, 0])
        qb = torch.zeros_like(a[:, 0])
        for t in range(a.shape[1] - 1, -1, -1):
            qa = a[:, t] * (gA[:, t] + qa)
            qb = a[:, t] * (gB[:, t] + qb)
            P = a[:, t] * P
        return torch.stack([P, qa, qb])

    def linear_bwd_fixup(self, a, b, carries, yin, gA, gB):
        A, Bv = carries[0].to(a.dtype), carries[1].to(a.dtype)
        prev = []
        for t in range(a.shape[1]):
            prev.append((A, Bv))
            A = a[:, t] * A
            Bv = a[:, t] * Bv + b[:, t]
        ya, yb = yin[0].to(a.dtype), yin[1].to(a.dtype)
        da, db = torch.empty_like(a), torch.empty_like(b)
        for t in range(a.shape[1] - 1, -1, -1):
            GA, GB = gA[:, t] + ya, gB[:, t] + yb
            da[:, t] = GA * prev[t][0] + GB * prev[t][1]
            db[:, t] = GB
            ya, yb = a[:, t] * GA, a[:, t] * GB
        return da, db

    # ---- parallel_scan_log: x_t = logaddexp(x_{t-1} + lc_t, lv_{t+1})
    def log_carry_fwd(self, lc, lv):
        alpha = lc.sum(1)
        x = torch.full_like(lc[:, 0], float("-inf"))
        for t in range(lc.shape[1]):
            x = torch.logaddexp(x + lc[:, t], lv[:, t + 1])
        return torch.stack([alpha, x])

    def log_fwd_fixup(self, lc, lv, lh_in):
        x = lh_in.to(lc.dtype)
        hs = []
        for t in range(lc.shape[1]):
            x = torch.logaddexp(x + lc[:, t], lv[:, t + 1])
            hs.append(torch.exp(x))
        return torch.stack(hs, 1), lh_in.clone()

    def log_carry_bwd(self, lc, gh):
        P = torch.ones_like(lc[:, 0])
        Q = torch.zeros_like(lc[:, 0])
        for t in range(lc.shape[1] - 1, -1, -1):
            a = torch.exp(lc[:, t])
            Q = a * (gh[:, t] + Q)
            P = a * P
        return torch.stack([P, Q])

    def log_bwd_fixup(self, lc, lv, lh_in, carries, yin, gh):
        x = lh_in.to(lc.dtype)
        prev = []
        for t in range(lc.shape[1]):
            prev.append(x)
            x = torch.logaddexp(x + lc[:, t], lv[:, t + 1])
        y = yin.to(lc.dtype)
        dlc, dlv = torch.empty_like(lc), torch.empty_like(lv)
        for t in range(lc.shape[1] - 1, -1, -1):
            G = gh[:, t] + y
            dlc[:, t] = G * torch.exp(lc[:, t] + prev[t])
            dlv[:, t + 1] = G * torch.exp(lv[:, t + 1])
            y = torch.exp(lc[:, t]) * G
        dlv[:, 0] = y * torch.exp(lh_in.to(lc.dtype))
        return dlc, dlv
