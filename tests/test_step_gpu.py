"""GPU parity of the fused per-token step kernels (the streaming path).

* Against the reference: each mixer's step() over a few tokens, from the
  reference module's weights (tests/golden/step_*.npz, made by
  tests/golden/make_golden.py from MinGRU.step ... DeltaMinGRU.step,
  min_gru.py:1399-1448, 1858-1901, 2316-2359, 2776-2818, 3611-3688), with
  and without decay; fp64 references, fp32 here (projections included), so
  rtol 1e-4 / atol 1e-4 as for the module fixtures.
* Each kernel against a plain PyTorch fp32 restatement of the same update,
  at fp32 (rtol 1e-5 / atol 1e-6) and bf16 storage (rtol 2e-2 / atol 2e-2).
* The C ABI's in-place form (new state over the previous one)."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden

pytestmark = pytest.mark.gpu

FWD = dict(rtol=1e-5, atol=1e-6)
HALF = dict(rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("name", golden_names("step_"))
def test_step_matches_reference(cuda, name):
    import mingru_b200 as mb

    g = load_golden(name)
    meta = json.loads(str(g["meta"]))
    mod = getattr(mb, meta["cls"])(**meta["kwargs"])
    mod.load_state_dict({k[3:]: torch.from_numpy(v) for k, v in g.items() if k.startswith("sd.")})
    mod = mod.float().to(cuda)
    xs = torch.as_tensor(g["x"], dtype=torch.float32, device=cuda)
    dts = torch.as_tensor(g["delta_t"], dtype=torch.float32, device=cuda) if "delta_t" in g else None
    h, ys, hs = None, [], []
    for t in range(xs.shape[1]):
        r = mod.step(xs[:, t], h, None if dts is None else dts[:, t])
        if meta["cls"] == "DeltaMinGRU":
            y, h = r
        else:
            y = h = r
        ys.append(y)
        hs.append(h)
    mb.raise_device_error(cuda)
    tol = dict(rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(torch.stack(ys, 1).double().cpu().numpy(), g["y"], **tol)
    np.testing.assert_allclose(torch.stack(hs, 1).double().cpu().numpy(), g["h"], **tol)


def _g(x):
    return torch.where(x >= 0, x + 0.5, torch.sigmoid(x))


def _givens_ref(theta, v, R, k):
    v = v.clone()
    for r in range(R):
        for m in range(k // 2):
            a = (r % 2 + 2 * m) % k
            b = (a + 1) % k
            c, s = torch.cos(theta[:, :, r, m]), torch.sin(theta[:, :, r, m])
            va, vb = v[..., a].clone(), v[..., b].clone()
            v[..., a] = c * va - s * vb
            v[..., b] = s * va + c * vb
    return v


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_kernels_vs_torch(cuda, dtype):
    from mingru_b200 import step_ops as so

    tol = FWD if dtype == torch.float32 else HALF
    gen = torch.Generator(device=cuda).manual_seed(5)
    r = lambda *s: torch.randn(*s, device=cuda, generator=gen)
    B, D, n = 7, 96, 40
    c = lambda t: t.to(dtype)
    f = lambda t: t.to(dtype).float()

    k, xh, hp, gm = r(B, D), r(B, D), r(B, D), torch.rand(B, D, device=cuda, generator=gen)
    ref = gm.to(dtype).float() * (1 - torch.sigmoid(f(k))) * f(hp) + torch.sigmoid(f(k)) * _g(f(xh))
    torch.testing.assert_close(so.mingru_step(c(k), c(xh), c(hp), c(gm)).float(), ref, **tol)
    ref0 = (1 - torch.sigmoid(f(k))) * f(hp) + torch.sigmoid(f(k)) * _g(f(xh))
    torch.testing.assert_close(so.mingru_step(c(k), c(xh), c(hp)).float(), ref0, **tol)

    z, s = r(B, D), r(B, D)
    for coupled in (False, True):
        a = torch.tanh(f(s)) * ((1 - torch.sigmoid(f(z))) if coupled else 1.0) * f(gm)
        ref = a * f(hp) + torch.sigmoid(f(z)) * f(xh)
        got = so.signed_step(c(z), c(s), c(xh), c(hp), c(gm), coupled)
        torch.testing.assert_close(got.float(), ref, **tol)

    th, u, gb = r(B, n), r(B, n), torch.rand(B, n, device=cuda, generator=gen)
    z2, x2, h2 = r(B, 2 * n), r(B, 2 * n), r(B, 2 * n)
    v = f(h2).view(B, n, 2)
    cs, sn, d = torch.cos(f(th)), torch.sin(f(th)), torch.tanh(f(u))
    v1 = d * v[..., 1]
    out = torch.stack([cs * v[..., 0] - sn * v1, sn * v[..., 0] + cs * v1], -1) * f(gb)[..., None]
    ref = (out + (torch.sigmoid(f(z2)) * f(x2)).view(B, n, 2)).view(B, 2 * n)
    torch.testing.assert_close(so.rotation_step(c(th), c(u), c(z2), c(x2), c(h2), c(gb)).float(),
                               ref, **tol)

    for kk, R in ((4, 2), (8, 3), (16, 1)):
        nb = 12
        thg = r(B, nb, R, kk // 2)
        zg, xg, hg = r(B, nb * kk), r(B, nb * kk), r(B, nb * kk)
        gg = torch.rand(B, nb, device=cuda, generator=gen)
        v = _givens_ref(f(thg), f(hg).view(B, nb, kk), R, kk) * f(gg)[..., None]
        ref = (v + (torch.sigmoid(f(zg)) * f(xg)).view(B, nb, kk)).view(B, nb * kk)
        got = so.givens_step(c(thg), c(zg), c(xg), c(hg), c(gg))
        torch.testing.assert_close(got.float(), ref, **tol)

    H, nh, dk, dv = 3, 2, 16, 24
    q = r(B, H, dk)
    kd = torch.nn.functional.normalize(r(B, H, nh, dk), dim=-1)
    vd = r(B, H, nh, dv)
    bd = 2 * torch.sigmoid(r(B, H, nh))
    gd = torch.rand(B, H, device=cuda, generator=gen)
    Hp = r(B, H, dk, dv) * 0.3
    Hr = f(Hp) * f(gd)[..., None, None]
    for m in range(nh):
        km, vm = f(kd[:, :, m]), f(vd[:, :, m])
        kH = torch.einsum("bhk,bhkv->bhv", km, Hr)
        Hr = Hr + f(bd[:, :, m])[..., None, None] * torch.einsum("bhk,bhv->bhkv", km, vm - kH)
    yr = torch.einsum("bhk,bhkv->bhv", f(q), Hr)
    y, Hn = so.delta_step(c(q), c(kd), c(vd), c(bd), c(Hp), c(gd))
    torch.testing.assert_close(y.float(), yr, **tol)
    torch.testing.assert_close(Hn.float(), Hr, **tol)


def test_in_place_state(cuda):
    """The C ABI lets the new state overwrite the previous one."""
    import mingru_b200 as mb
    from mingru_b200 import _lib

    lib = _lib.load()
    gen = torch.Generator(device=cuda).manual_seed(9)
    k, xh, h = (torch.randn(4, 64, device=cuda, generator=gen) for _ in range(3))
    expect = (1 - torch.sigmoid(k)) * h + torch.sigmoid(k) * _g(xh)
    st = lib.mgs_mingru_step(k.data_ptr(), xh.data_ptr(), h.data_ptr(), None, h.data_ptr(), 4, 64,
                             0, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.testing.assert_close(h, expect, **FWD)
    B, H, dk, dv = 2, 2, 8, 8
    q = torch.randn(B, H, dk, device=cuda, generator=gen)
    kd = torch.nn.functional.normalize(torch.randn(B, H, 1, dk, device=cuda, generator=gen), dim=-1)
    vd = torch.randn(B, H, 1, dv, device=cuda, generator=gen)
    bd = torch.rand(B, H, 1, device=cuda, generator=gen)
    Hs = torch.randn(B, H, dk, dv, device=cuda, generator=gen)
    y_ref, H_ref = mb.step_ops.delta_step(q, kd, vd, bd, Hs.clone())
    y = torch.empty(B, H, dv, device=cuda)
    st = lib.mgs_delta_step(q.data_ptr(), kd.data_ptr(), vd.data_ptr(), bd.data_ptr(), None,
                            Hs.data_ptr(), y.data_ptr(), Hs.data_ptr(), B, H, 1, dk, dv, 0,
                            torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.testing.assert_close(Hs, H_ref, **FWD)
    torch.testing.assert_close(y, y_ref, **FWD)
