"""GPU parity of the drop-in modules: each reference module's state_dict is
loaded into the mingru_b200 module, which must reproduce the reference's
output and the gradients w.r.t. the input and every parameter (golden
fixtures from the reference in fp64; here fp32 end to end, so the gate is
rtol 1e-4 / atol 1e-4 on outputs and 5e-4 on gradients -- the projections,
LayerNorms and MLPs around the scans add their own fp32 rounding). Also
checks that the parallel forward equals a loop of step() calls."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", golden_names("module_"))
def test_module_matches_reference(cuda, name):
    import mingru_b200 as mb

    g = load_golden(name)
    meta = json.loads(str(g["meta"]))
    mod = getattr(mb, meta["cls"])(**meta["kwargs"])
    mod.load_state_dict({k[3:]: torch.from_numpy(v) for k, v in g.items() if k.startswith("sd.")})
    mod = mod.float().to(cuda)
    x = torch.as_tensor(g["x"], dtype=torch.float32, device=cuda).requires_grad_(True)
    if meta["cls"] == "MinGRUStack":
        out, _ = mod(x)
    elif meta["cls"] == "DeltaMinGRU" and "delta_t" not in g:
        out = mod(x)
    else:
        dt = torch.as_tensor(g["delta_t"], dtype=torch.float32, device=cuda) if "delta_t" in g else None
        out = mod(x, None, dt)
    np.testing.assert_allclose(out.detach().double().cpu().numpy(), g["out"], rtol=1e-4, atol=1e-4)
    (out * torch.as_tensor(g["cot"], dtype=torch.float32, device=cuda)).sum().backward()
    mb.raise_device_error(cuda)
    np.testing.assert_allclose(x.grad.double().cpu().numpy(), g["dx"], rtol=5e-4, atol=5e-4)
    for pn, p in mod.named_parameters():
        got = p.grad.double().cpu().numpy() if p.grad is not None else np.zeros(p.shape)
        np.testing.assert_allclose(got, g["grad." + pn], rtol=5e-4, atol=5e-4, err_msg=pn)


MIXERS = [
    ("MinGRU", dict(learnable_h0=True)),
    ("SignedMinGRU", dict(coupled=True)),
    ("RotationMinGRU", dict()),
    ("GivensMinGRU", dict(block_size=8, rounds=3)),
    ("DeltaMinGRU", dict(n_heads=2, chunk_size=16)),
]


@pytest.mark.parametrize("cls,kw", MIXERS)
def test_forward_equals_step_loop(cuda, cls, kw):
    import mingru_b200 as mb

    torch.manual_seed(0)
    mod = getattr(mb, cls)(8, 32, **kw).to(cuda)
    x = torch.randn(2, 45, 8, device=cuda)
    with torch.no_grad():
        full = mod(x)
        h = None
        outs = []
        for t in range(x.shape[1]):
            r = mod.step(x[:, t], h)
            if cls == "DeltaMinGRU":
                y_t, h = r
            else:
                y_t = h = r
            outs.append(y_t)
        stepped = torch.stack(outs, 1)
    torch.testing.assert_close(full, stepped, rtol=1e-4, atol=1e-4)


def test_chunked_equals_full(cuda):
    """Carrying the last state into a second forward equals one long forward."""
    import mingru_b200 as mb

    torch.manual_seed(1)
    stack = mb.MinGRUStack(8, 16, 3, mixer=["log", "signed", "rotation"]).to(cuda)
    x = torch.randn(2, 60, 8, device=cuda)
    with torch.no_grad():
        full, _ = stack(x)
        a, st = stack(x[:, :25])
        b, _ = stack(x[:, 25:], st)
    torch.testing.assert_close(torch.cat([a, b], 1), full, rtol=1e-4, atol=1e-4)
