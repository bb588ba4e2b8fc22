"""The public scan ops, backed only by the sm_100a kernels of ``libmingru_scan.so``.

Drop-in replacements for the reference's four public scan functions
(``parallel_scan_log``, ``linear_scan``, ``matrix_scan``,
``matrix_affine_scan``; reference ``src/mingru/min_gru.py:755, 1454, 1513,
1584``) and for its two module fast paths (``angle_scan_impl``,
``delta_scan_impl``; reference ``src/mingru/triton_scans.py:1743, 2403``):
same argument order, shapes, dtypes and return values. What the reference's
``MINGRU_SCAN`` seam did (``min_gru.py:85-704``: choose Triton or eager per
call, warn, fall back) does not exist here: the ops always run the CUDA
kernels, raise ``ValueError`` for CPU tensors or inputs outside the kernels'
envelope, and ``RuntimeError`` for device-side failures.

Each op is a ``torch.library.custom_op`` with a registered fake (shape)
function and a ``register_autograd`` backward that calls the op's own
backward kernel, so ``torch.compile`` sees opaque ops (the reference wires
its Triton ops the same way, ``triton_scans.py:1465-1552``). Second-order
autograd is not supported and raises, as in the reference
(``triton_scans.py:1523-1532``).
"""

from __future__ import annotations

import torch

from . import _lib

_DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _dtype_code(op: str, t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODES[t.dtype]
    except KeyError:
        raise ValueError(
            f"{op}: dtype {t.dtype} is not supported (float32, bfloat16, float16; "
            "arithmetic is always fp32)"
        ) from None


def _require_cuda(op: str, *ts: torch.Tensor) -> None:
    dev = ts[0].device
    for t in ts:
        if not t.is_cuda:
            raise ValueError(
                f"{op}: expected CUDA tensors (this library has no CPU path), got {t.device}"
            )
        if t.device != dev:
            raise ValueError(f"{op}: tensors on different devices ({dev} vs {t.device})")


def _dense(t: torch.Tensor) -> torch.Tensor:
    """C-contiguous with a 16-byte aligned base (what the vector loads need)."""
    t = t.contiguous()
    if t.data_ptr() % 16 != 0:
        t = t.clone()
    return t


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def take_device_error(device=None) -> int:
    """Synchronise and return/clear the sticky device error bits (0 = clean).

    A look-back wait that exhausts its bound records ``MGS_LOOKBACK_TIMEOUT``
    there instead of hanging; call this after a step to turn such a record
    into an exception (see ``raise_device_error``).
    """
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    with torch.cuda.device(device):
        return int(_lib.load().mgs_take_device_error(torch.cuda.current_stream(device).cuda_stream))


def raise_device_error(device=None) -> None:
    bits = take_device_error(device)
    if bits:
        names = [n for s, n in _lib.STATUS_NAMES.items() if s and bits & (1 << s)]
        raise RuntimeError(f"scan kernels reported device errors: {', '.join(names)}")


# =========================================================== linear_scan ==


@torch.library.custom_op("mingru_b200::linear_scan_fwd", mutates_args=())
def _linear_scan_fwd(
    a: torch.Tensor, b: torch.Tensor, save_carries: bool
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(a.device):  # sizes are queried on the launch device
        a, b = _dense(a), _dense(b)
        Bn, T, D = a.shape
        code = _dtype_code("linear_scan", a)
        A, Bc = torch.empty_like(a), torch.empty_like(b)
        csz = lib.mgs_linear_scan_carry_size(Bn, T, D, code) if save_carries else 0
        carries = torch.empty(csz // 4, dtype=torch.float32, device=a.device)
        ws = _workspace(lib.mgs_linear_scan_workspace_size(Bn, T, D, code), a.device)
        st = lib.mgs_linear_scan_fwd(
            _ptr(a), _ptr(b), _ptr(A), _ptr(Bc), _ptr(carries) if save_carries else None,
            Bn, T, D, code, _ptr(ws), ws.numel(), _stream(a),
        )
        _lib.check(st, "linear_scan forward")
        return A, Bc, carries


@_linear_scan_fwd.register_fake
def _(a, b, save_carries):
    Bn, T, D = a.shape
    csz = _lib.load().mgs_linear_scan_carry_size(Bn, T, D, _dtype_code("linear_scan", a))
    n = csz // 4 if save_carries else 0
    return torch.empty_like(a), torch.empty_like(b), a.new_empty((n,), dtype=torch.float32)


@torch.library.custom_op("mingru_b200::linear_scan_bwd", mutates_args=())
def _linear_scan_bwd(
    a: torch.Tensor, b: torch.Tensor, gA: torch.Tensor, gBc: torch.Tensor, carries: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(a.device):  # sizes are queried on the launch device
        a, b, gA, gBc = (_dense(x) for x in (a, b, gA.to(a.dtype), gBc.to(a.dtype)))
        Bn, T, D = a.shape
        code = _dtype_code("linear_scan", a)
        if carries.numel() * 4 < lib.mgs_linear_scan_carry_size(Bn, T, D, code):
            raise RuntimeError("linear_scan backward: forward carries were not saved")
        da, db = torch.empty_like(a), torch.empty_like(b)
        ws = _workspace(lib.mgs_linear_scan_workspace_size(Bn, T, D, code), a.device)
        st = lib.mgs_linear_scan_bwd(
            _ptr(a), _ptr(b), _ptr(gA), _ptr(gBc), _ptr(carries), _ptr(da), _ptr(db),
            Bn, T, D, code, _ptr(ws), ws.numel(), _stream(a),
        )
        _lib.check(st, "linear_scan backward")
        return da, db


@_linear_scan_bwd.register_fake
def _(a, b, gA, gBc, carries):
    return torch.empty_like(a), torch.empty_like(b)


def _linear_setup(ctx, inputs, output):
    a, b, _ = inputs
    ctx.save_for_backward(a, b, output[2])
    ctx.mark_non_differentiable(output[2])
    ctx.set_materialize_grads(False)


def _linear_backward(ctx, gA, gBc, _gcarries):
    if torch.is_grad_enabled():
        raise RuntimeError("linear_scan does not support second-order autograd (create_graph=True)")
    a, b, carries = ctx.saved_tensors
    if gA is None:
        gA = torch.zeros_like(a)
    if gBc is None:
        gBc = torch.zeros_like(a)
    da, db = _linear_scan_bwd(a, b, gA, gBc, carries)
    return da, db, None


torch.library.register_autograd(
    "mingru_b200::linear_scan_fwd", _linear_backward, setup_context=_linear_setup
)


def linear_scan(a: torch.Tensor, b: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Scan ``h_t = a_t h_{t-1} + b_t`` over ``dim=1``; returns ``(A, Bc)``.

    ``a``, ``b``: ``(B, T, D)`` CUDA tensors of one dtype (float32, bfloat16 or
    float16). ``A_t = prod_{s<=t} a_s`` and ``Bc_t`` is the ``h_0 = 0``
    solution, so ``h_t = A_t h_0 + Bc_t``; outputs have the input dtype,
    arithmetic is fp32. Same contract as the reference's
    ``min_gru.linear_scan`` (``min_gru.py:1454-1510``).
    """
    op = "linear_scan"
    if a.ndim != 3 or b.ndim != 3 or a.shape != b.shape:
        raise ValueError(
            f"{op}: need matching (B, T, D) a and b (got a={tuple(a.shape)}, b={tuple(b.shape)})"
        )
    _require_cuda(op, a, b)
    if a.dtype != b.dtype:
        raise ValueError(f"{op}: a and b must share a dtype ({a.dtype} vs {b.dtype})")
    _dtype_code(op, a)
    need = torch.is_grad_enabled() and (a.requires_grad or b.requires_grad)
    A, Bc, _ = _linear_scan_fwd(a, b, need)
    return A, Bc


# ===================================================== parallel_scan_log ==


@torch.library.custom_op("mingru_b200::log_scan_fwd", mutates_args=())
def _log_scan_fwd(
    log_coeffs: torch.Tensor, log_values: torch.Tensor, save_carries: bool
) -> tuple[torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(log_coeffs.device):  # sizes are queried on the launch device
        lc, lv = _dense(log_coeffs), _dense(log_values)
        Bn, T, D = lc.shape
        code = _dtype_code("parallel_scan_log", lc)
        h = torch.empty_like(lc)
        csz = lib.mgs_log_scan_carry_size(Bn, T, D, code) if save_carries else 0
        carries = torch.empty(csz // 4, dtype=torch.float32, device=lc.device)
        ws = _workspace(lib.mgs_log_scan_workspace_size(Bn, T, D, code), lc.device)
        st = lib.mgs_log_scan_fwd(
            _ptr(lc), _ptr(lv), _ptr(h), _ptr(carries) if save_carries else None,
            Bn, T, D, code, _ptr(ws), ws.numel(), _stream(lc),
        )
        _lib.check(st, "parallel_scan_log forward")
        return h, carries


@_log_scan_fwd.register_fake
def _(log_coeffs, log_values, save_carries):
    Bn, T, D = log_coeffs.shape
    csz = _lib.load().mgs_log_scan_carry_size(Bn, T, D, _dtype_code("parallel_scan_log", log_coeffs))
    n = csz // 4 if save_carries else 0
    return torch.empty_like(log_coeffs), log_coeffs.new_empty((n,), dtype=torch.float32)


@torch.library.custom_op("mingru_b200::log_scan_bwd", mutates_args=())
def _log_scan_bwd(
    log_coeffs: torch.Tensor, log_values: torch.Tensor, grad_h: torch.Tensor, carries: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(log_coeffs.device):  # sizes are queried on the launch device
        lc, lv = _dense(log_coeffs), _dense(log_values)
        gh = _dense(grad_h.to(lc.dtype))
        Bn, T, D = lc.shape
        code = _dtype_code("parallel_scan_log", lc)
        if carries.numel() * 4 < lib.mgs_log_scan_carry_size(Bn, T, D, code):
            raise RuntimeError("parallel_scan_log backward: forward carries were not saved")
        dlc, dlv = torch.empty_like(lc), torch.empty_like(lv)
        ws = _workspace(lib.mgs_log_scan_workspace_size(Bn, T, D, code), lc.device)
        st = lib.mgs_log_scan_bwd(
            _ptr(lc), _ptr(lv), _ptr(gh), _ptr(carries), _ptr(dlc), _ptr(dlv),
            Bn, T, D, code, _ptr(ws), ws.numel(), _stream(lc),
        )
        _lib.check(st, "parallel_scan_log backward")
        return dlc, dlv


@_log_scan_bwd.register_fake
def _(log_coeffs, log_values, grad_h, carries):
    return torch.empty_like(log_coeffs), torch.empty_like(log_values)


def _log_setup(ctx, inputs, output):
    lc, lv, _ = inputs
    ctx.save_for_backward(lc, lv, output[1])
    ctx.mark_non_differentiable(output[1])
    ctx.set_materialize_grads(False)


def _log_backward(ctx, grad_h, _gcarries):
    if torch.is_grad_enabled():
        raise RuntimeError(
            "parallel_scan_log does not support second-order autograd (create_graph=True)"
        )
    lc, lv, carries = ctx.saved_tensors
    if grad_h is None:
        return None, None, None
    dlc, dlv = _log_scan_bwd(lc, lv, grad_h, carries)
    return dlc, dlv, None


torch.library.register_autograd("mingru_b200::log_scan_fwd", _log_backward, setup_context=_log_setup)


def parallel_scan_log(log_coeffs: torch.Tensor, log_values: torch.Tensor) -> torch.Tensor:
    """Heinsen log-space scan: ``h_t = a_t h_{t-1} + b_t`` given logs.

    ``log_coeffs`` ``(B, T, D)`` holds ``log a_t``; ``log_values``
    ``(B, T+1, D)`` holds ``log h_0`` in slot 0 and ``log b_t`` after it.
    Returns ``h_1..h_T`` as ``(B, T, D)`` in the input dtype (fp32 maths).
    Same contract as the reference's ``min_gru.parallel_scan_log``
    (``min_gru.py:755-807``).
    """
    op = "parallel_scan_log"
    lc, lv = log_coeffs, log_values
    if lc.ndim != 3 or lv.ndim != 3 or tuple(lv.shape) != (lc.shape[0], lc.shape[1] + 1, lc.shape[2]):
        raise ValueError(
            f"{op}: need (B, T, D) log_coeffs and (B, T+1, D) log_values "
            f"(got log_coeffs={tuple(lc.shape)}, log_values={tuple(lv.shape)})"
        )
    _require_cuda(op, lc, lv)
    if lc.dtype != lv.dtype:
        raise ValueError(f"{op}: log_coeffs and log_values must share a dtype ({lc.dtype} vs {lv.dtype})")
    _dtype_code(op, lc)
    need = torch.is_grad_enabled() and (lc.requires_grad or lv.requires_grad)
    h, _ = _log_scan_fwd(lc, lv, need)
    return h


# =================================================== MinGRU gate scan ==


@torch.library.custom_op("mingru_b200::log_gate_scan_fwd", mutates_args=())
def _log_gate_fwd(
    k: torch.Tensor, x: torch.Tensor, log_h0: torch.Tensor, save_carries: bool
) -> tuple[torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(k.device):  # sizes are queried on the launch device
        k, x, lh0 = _dense(k), _dense(x), _dense(log_h0)
        Bn, T, D = k.shape
        code = _dtype_code("mingru_gate_scan", k)
        h = torch.empty_like(k)
        csz = lib.mgs_log_gate_scan_carry_size(Bn, T, D, code) if save_carries else 0
        carries = torch.empty(csz // 4, dtype=torch.float32, device=k.device)
        ws = _workspace(lib.mgs_log_gate_scan_workspace_size(Bn, T, D, code), k.device)
        st = lib.mgs_log_gate_scan_fwd(
            _ptr(k), _ptr(x), _ptr(lh0), _ptr(h), _ptr(carries) if save_carries else None,
            Bn, T, D, code, _ptr(ws), ws.numel(), _stream(k),
        )
        _lib.check(st, "mingru_gate_scan forward")
        return h, carries


@_log_gate_fwd.register_fake
def _(k, x, log_h0, save_carries):
    Bn, T, D = k.shape
    csz = _lib.load().mgs_log_gate_scan_carry_size(Bn, T, D, _dtype_code("mingru_gate_scan", k))
    return torch.empty_like(k), k.new_empty((csz // 4 if save_carries else 0,), dtype=torch.float32)


@torch.library.custom_op("mingru_b200::log_gate_scan_bwd", mutates_args=())
def _log_gate_bwd(
    k: torch.Tensor, x: torch.Tensor, log_h0: torch.Tensor, grad_h: torch.Tensor,
    carries: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(k.device):  # sizes are queried on the launch device
        k, x, lh0 = _dense(k), _dense(x), _dense(log_h0)
        gh = _dense(grad_h.to(k.dtype))
        Bn, T, D = k.shape
        code = _dtype_code("mingru_gate_scan", k)
        if carries.numel() * 4 < lib.mgs_log_gate_scan_carry_size(Bn, T, D, code):
            raise RuntimeError("mingru_gate_scan backward: forward carries were not saved")
        dk, dx, dlh0 = torch.empty_like(k), torch.empty_like(x), torch.empty_like(lh0)
        ws = _workspace(lib.mgs_log_gate_scan_workspace_size(Bn, T, D, code), k.device)
        st = lib.mgs_log_gate_scan_bwd(
            _ptr(k), _ptr(x), _ptr(lh0), _ptr(gh), _ptr(carries), _ptr(dk), _ptr(dx), _ptr(dlh0),
            Bn, T, D, code, _ptr(ws), ws.numel(), _stream(k),
        )
        _lib.check(st, "mingru_gate_scan backward")
        return dk, dx, dlh0


@_log_gate_bwd.register_fake
def _(k, x, log_h0, grad_h, carries):
    return torch.empty_like(k), torch.empty_like(x), torch.empty_like(log_h0)


def _log_gate_setup(ctx, inputs, output):
    k, x, lh0, _ = inputs
    ctx.save_for_backward(k, x, lh0, output[1])
    ctx.mark_non_differentiable(output[1])
    ctx.set_materialize_grads(False)


def _log_gate_backward(ctx, grad_h, _gcarries):
    if torch.is_grad_enabled():
        raise RuntimeError(
            "mingru_gate_scan does not support second-order autograd (create_graph=True)"
        )
    k, x, lh0, carries = ctx.saved_tensors
    if grad_h is None:
        return None, None, None, None
    dk, dx, dlh0 = _log_gate_bwd(k, x, lh0, grad_h, carries)
    return dk, dx, dlh0, None


torch.library.register_autograd(
    "mingru_b200::log_gate_scan_fwd", _log_gate_backward, setup_context=_log_gate_setup
)


def mingru_gate_scan(k: torch.Tensor, x: torch.Tensor, log_h0: torch.Tensor) -> torch.Tensor:
    """MinGRU's scan straight from its pre-activations: returns ``h_1..h_T``.

    ``k`` = ``linear_z(x)`` and ``x`` = ``linear_h(x)`` (the candidate
    pre-activation), both ``(B, T, D)``; ``log_h0`` ``(B, D)`` or ``(B, 1, D)``.
    Equal to ``parallel_scan_log(-softplus(k), cat([log_h0, -softplus(-k) +
    log_g(x)], 1))`` -- what MinGRU.forward builds without decay (reference
    ``min_gru.py:1383-1397``) -- with the prologue fused into the scan kernels:
    the log coefficients never exist in HBM on the column path (fp32,
    T <= 1024), and the backward returns ``dk``, ``dx`` and ``dlog_h0``
    directly. Differentiable w.r.t. all three inputs.
    """
    op = "mingru_gate_scan"
    if k.ndim != 3 or x.shape != k.shape:
        raise ValueError(f"{op}: need matching (B, T, D) k and x (got k={tuple(k.shape)}, "
                         f"x={tuple(x.shape)})")
    Bn, T, D = k.shape
    lh0 = log_h0.reshape(Bn, D) if log_h0.ndim == 3 and log_h0.shape[1] == 1 else log_h0
    if tuple(lh0.shape) != (Bn, D):
        raise ValueError(f"{op}: log_h0 must be (B, D) or (B, 1, D) (got {tuple(log_h0.shape)})")
    _require_cuda(op, k, x, lh0)
    if x.dtype != k.dtype or lh0.dtype != k.dtype:
        raise ValueError(f"{op}: k, x and log_h0 must share a dtype")
    _dtype_code(op, k)
    need = torch.is_grad_enabled() and (k.requires_grad or x.requires_grad or lh0.requires_grad)
    h, _ = _log_gate_fwd(k, x, lh0, need)
    return h


# ================================================ matrix(_affine)_scan ==


@torch.library.custom_op("mingru_b200::affine_scan_fwd", mutates_args=())
def _affine_scan_fwd(
    A: torch.Tensor, Bm: torch.Tensor, save_carries: bool
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(A.device):  # sizes are queried on the launch device
        A, Bm = _dense(A), _dense(Bm)
        Bn, T, n, k, _ = A.shape
        v = Bm.shape[-1]
        code = _dtype_code("matrix_affine_scan", A)
        Abar, Bbar = torch.empty_like(A), torch.empty_like(Bm)
        csz = lib.mgs_affine_scan_carry_size(Bn, T, n, k, v, code) if save_carries else 0
        carries = torch.empty(csz // 4, dtype=torch.float32, device=A.device)
        ws = _workspace(lib.mgs_affine_scan_workspace_size(Bn, T, n, k, v, code), A.device)
        st = lib.mgs_affine_scan_fwd(
            _ptr(A), _ptr(Bm), _ptr(Abar), _ptr(Bbar), _ptr(carries) if csz else None,
            Bn, T, n, k, v, code, _ptr(ws), ws.numel(), _stream(A),
        )
        _lib.check(st, "matrix_affine_scan forward")
        return Abar, Bbar, carries


@_affine_scan_fwd.register_fake
def _(A, Bm, save_carries):
    Bn, T, n, k, _ = A.shape
    v = Bm.shape[-1]
    csz = _lib.load().mgs_affine_scan_carry_size(Bn, T, n, k, v, _dtype_code("matrix_affine_scan", A))
    nfl = csz // 4 if save_carries else 0
    return torch.empty_like(A), torch.empty_like(Bm), A.new_empty((nfl,), dtype=torch.float32)


@torch.library.custom_op("mingru_b200::affine_scan_bwd", mutates_args=())
def _affine_scan_bwd(
    A: torch.Tensor, Bm: torch.Tensor, Abar: torch.Tensor, Bbar: torch.Tensor,
    gAbar: torch.Tensor, gBbar: torch.Tensor, carries: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(A.device):  # sizes are queried on the launch device
        A, Bm, Abar, Bbar = (_dense(x) for x in (A, Bm, Abar, Bbar))
        gA, gB = _dense(gAbar.to(A.dtype)), _dense(gBbar.to(A.dtype))
        Bn, T, n, k, _ = A.shape
        v = Bm.shape[-1]
        code = _dtype_code("matrix_affine_scan", A)
        csz = lib.mgs_affine_scan_carry_size(Bn, T, n, k, v, code)
        if carries.numel() * 4 < csz:
            raise RuntimeError("matrix_affine_scan backward: forward carries were not saved")
        dA, dB = torch.empty_like(A), torch.empty_like(Bm)
        ws = _workspace(lib.mgs_affine_scan_workspace_size(Bn, T, n, k, v, code), A.device)
        st = lib.mgs_affine_scan_bwd(
            _ptr(A), _ptr(Bm), _ptr(Abar), _ptr(Bbar), _ptr(gA), _ptr(gB),
            _ptr(carries) if csz else None, _ptr(dA), _ptr(dB),
            Bn, T, n, k, v, code, _ptr(ws), ws.numel(), _stream(A),
        )
        _lib.check(st, "matrix_affine_scan backward")
        return dA, dB


@_affine_scan_bwd.register_fake
def _(A, Bm, Abar, Bbar, gAbar, gBbar, carries):
    return torch.empty_like(A), torch.empty_like(Bm)


def _affine_setup(ctx, inputs, output):
    A, Bm, _ = inputs
    Abar, Bbar, carries = output
    ctx.save_for_backward(A, Bm, Abar, Bbar, carries)
    ctx.mark_non_differentiable(carries)
    ctx.set_materialize_grads(False)


def _affine_backward(ctx, gAbar, gBbar, _gcarries):
    if torch.is_grad_enabled():
        raise RuntimeError(
            "matrix_affine_scan does not support second-order autograd (create_graph=True)"
        )
    A, Bm, Abar, Bbar, carries = ctx.saved_tensors
    if gAbar is None and gBbar is None:
        return None, None, None
    if gAbar is None:
        gAbar = torch.zeros_like(A)
    if gBbar is None:
        gBbar = torch.zeros_like(Bm)
    dA, dB = _affine_scan_bwd(A, Bm, Abar, Bbar, gAbar, gBbar, carries)
    return dA, dB, None


torch.library.register_autograd(
    "mingru_b200::affine_scan_fwd", _affine_backward, setup_context=_affine_setup
)

_MAX_KV = 64


def matrix_affine_scan(A: torch.Tensor, Bm: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Scan ``H_t = A_t H_{t-1} + B_t`` per block; returns ``(Abar, Bbar)``.

    ``A`` ``(B, T, n, k, k)`` and ``Bm`` ``(B, T, n, k, v)`` CUDA tensors of one
    dtype. ``Abar_t`` is the running product ``A_t ... A_1`` and ``Bbar_t``
    the ``H_0 = 0`` solution, so ``H_t = Abar_t H_0 + Bbar_t``. Same contract
    as the reference's ``min_gru.matrix_affine_scan`` (``min_gru.py:1584-1655``).
    """
    op = "matrix_affine_scan"
    if A.ndim != 5 or Bm.ndim != 5:
        raise ValueError(
            f"{op}: need 5-D (B, T, n, k, k) A and (B, T, n, k, v) Bm "
            f"(got A={tuple(A.shape)}, Bm={tuple(Bm.shape)})"
        )
    k, v = A.shape[-1], Bm.shape[-1]
    if A.shape[-2] != k or Bm.shape[-2] != k or A.shape[:3] != Bm.shape[:3]:
        raise ValueError(
            f"{op}: need a square A (A.shape[-2:] == (k, k)), Bm with k rows and A/Bm sharing "
            f"the (B, T, n) grid (got A={tuple(A.shape)}, Bm={tuple(Bm.shape)})"
        )
    if not (1 <= k <= _MAX_KV and 1 <= v <= _MAX_KV):
        raise ValueError(f"{op}: k and v must be in [1, {_MAX_KV}] (got k={k}, v={v})")
    _require_cuda(op, A, Bm)
    if A.dtype != Bm.dtype:
        raise ValueError(f"{op}: A and Bm must share a dtype ({A.dtype} vs {Bm.dtype})")
    _dtype_code(op, A)
    need = torch.is_grad_enabled() and (A.requires_grad or Bm.requires_grad)
    Abar, Bbar, _ = _affine_scan_fwd(A, Bm, need)
    return Abar, Bbar


def matrix_scan(M: torch.Tensor, b: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """2x2-block scan ``h_t = M_t h_{t-1} + b_t``; returns ``(A, Bc)``.

    ``M`` ``(B, T, n, 2, 2)``, ``b`` ``(B, T, n, 2)``; ``A`` is the running
    product and ``Bc`` the ``h_0 = 0`` solution. Same contract as the
    reference's ``min_gru.matrix_scan`` (``min_gru.py:1513-1581``); it is the
    ``k = 2, v = 1`` case of :func:`matrix_affine_scan`.
    """
    op = "matrix_scan"
    if M.ndim != 5 or b.ndim != 4 or M.shape[-2:] != (2, 2) or b.shape[-1] != 2 \
            or M.shape[:3] != b.shape[:3]:
        raise ValueError(
            f"{op}: need (B, T, n, 2, 2) M and (B, T, n, 2) b sharing the (B, T, n) grid "
            f"(got M={tuple(M.shape)}, b={tuple(b.shape)})"
        )
    Abar, Bbar = matrix_affine_scan(M, b.unsqueeze(-1))
    return Abar, Bbar.squeeze(-1)


# ====================================================== angle-fused scan ==


def brickwall_meta(rounds: int, k: int, device=None):
    """The (perm, sgn, p2p) plane metadata of the brick-wall layout that
    GivensMinGRU / RotationMinGRU build (reference ``min_gru.py:2544-2549``,
    ``2649-2678``, ``2202-2219``): round r pairs (i, i+1 mod k) for
    i = r%2, r%2+2, ...; sgn is -1 on i and +1 on i+1; p2p is the plane index."""
    perm = torch.empty(rounds, k, dtype=torch.int32)
    sgn = torch.empty(rounds, k, dtype=torch.float32)
    p2p = torch.empty(rounds, k, dtype=torch.int32)
    for r in range(rounds):
        i_idx = [(i % k) for i in range(r % 2, k, 2)]
        for m, i in enumerate(i_idx):
            j = (i + 1) % k
            perm[r, i], perm[r, j] = j, i
            sgn[r, i], sgn[r, j] = -1.0, 1.0
            p2p[r, i], p2p[r, j] = m, m
    if device is not None:
        perm, sgn, p2p = perm.to(device), sgn.to(device), p2p.to(device)
    return perm, sgn, p2p


def _is_brickwall(perm: torch.Tensor, sgn: torch.Tensor, p2p: torch.Tensor) -> bool:
    """Whether the metadata is the brick-wall layout. Checked once per tensor
    (one device-to-host copy) and remembered on the tensor object."""
    key = (perm._version, sgn._version, p2p._version, sgn.data_ptr(), p2p.data_ptr())
    memo = getattr(perm, "_mgs_brickwall", None)
    if memo is not None and memo[0] == key:
        return memo[1]
    R, k = perm.shape
    rp, rs, rq = brickwall_meta(R, k)
    ok = (torch.equal(perm.detach().cpu().to(torch.int32), rp)
          and torch.equal(sgn.detach().cpu().to(torch.float32), rs)
          and torch.equal(p2p.detach().cpu().to(torch.int32), rq))
    try:
        perm._mgs_brickwall = (key, ok)
    except (AttributeError, RuntimeError):
        pass
    return ok


@torch.library.custom_op("mingru_b200::angle_scan_fwd", mutates_args=())
def _angle_scan_fwd(
    theta: torch.Tensor, scale: torch.Tensor, gamma: torch.Tensor, b: torch.Tensor,
    h0: torch.Tensor, perm: torch.Tensor, sgn: torch.Tensor, p2p: torch.Tensor,
    has_scale: int, has_decay: int, brickwall: int, save_carries: bool,
) -> tuple[torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(theta.device):  # sizes are queried on the launch device
        theta, scale, gamma, b, h0 = (_dense(x) for x in (theta, scale, gamma, b, h0))
        Bn, T, n, R, half = theta.shape
        k = b.shape[-1]
        code = _dtype_code("angle_scan", b)
        h = torch.empty_like(b)
        csz = lib.mgs_angle_scan_carry_size(Bn, T, n, R, k, brickwall, code) if save_carries else 0
        carries = torch.empty(csz // 4, dtype=torch.float32, device=b.device)
        ws = _workspace(lib.mgs_angle_scan_workspace_size(Bn, T, n, R, k, brickwall, code), b.device)
        st = lib.mgs_angle_scan_fwd(
            _ptr(theta), _ptr(scale), _ptr(gamma), _ptr(b), _ptr(h0),
            _ptr(perm), _ptr(sgn), _ptr(p2p), _ptr(h), _ptr(carries) if csz else None,
            Bn, T, n, R, k, int(has_scale), int(has_decay), int(brickwall), code,
            _ptr(ws), ws.numel(), _stream(b),
        )
        _lib.check(st, "angle_scan forward")
        return h, carries


@_angle_scan_fwd.register_fake
def _(theta, scale, gamma, b, h0, perm, sgn, p2p, has_scale, has_decay, brickwall, save_carries):
    Bn, T, n, R, half = theta.shape
    k = b.shape[-1]
    csz = _lib.load().mgs_angle_scan_carry_size(Bn, T, n, R, k, brickwall, _dtype_code("angle_scan", b))
    return torch.empty_like(b), b.new_empty((csz // 4 if save_carries else 0,), dtype=torch.float32)


@torch.library.custom_op("mingru_b200::angle_scan_bwd", mutates_args=())
def _angle_scan_bwd(
    theta: torch.Tensor, scale: torch.Tensor, gamma: torch.Tensor, b: torch.Tensor,
    h0: torch.Tensor, perm: torch.Tensor, sgn: torch.Tensor, p2p: torch.Tensor,
    h: torch.Tensor, grad_h: torch.Tensor, carries: torch.Tensor,
    has_scale: int, has_decay: int, brickwall: int,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(theta.device):  # sizes are queried on the launch device
        theta, scale, gamma, b, h0, h = (_dense(x) for x in (theta, scale, gamma, b, h0, h))
        gh = _dense(grad_h.to(b.dtype))
        Bn, T, n, R, half = theta.shape
        k = b.shape[-1]
        code = _dtype_code("angle_scan", b)
        csz = lib.mgs_angle_scan_carry_size(Bn, T, n, R, k, brickwall, code)
        if carries.numel() * 4 < csz:
            raise RuntimeError("angle_scan backward: forward carries were not saved")
        dtheta, db, dh0 = torch.empty_like(theta), torch.empty_like(b), torch.empty_like(h0)
        dscale = torch.empty_like(scale) if has_scale else torch.zeros_like(scale)
        dgamma = torch.empty_like(gamma) if has_decay else torch.zeros_like(gamma)
        ws = _workspace(lib.mgs_angle_scan_workspace_size(Bn, T, n, R, k, brickwall, code), b.device)
        st = lib.mgs_angle_scan_bwd(
            _ptr(theta), _ptr(scale), _ptr(gamma), _ptr(b), _ptr(h0),
            _ptr(perm), _ptr(sgn), _ptr(p2p), _ptr(h), _ptr(gh), _ptr(carries) if csz else None,
            _ptr(dtheta), _ptr(dscale), _ptr(dgamma), _ptr(db), _ptr(dh0),
            Bn, T, n, R, k, int(has_scale), int(has_decay), int(brickwall), code,
            _ptr(ws), ws.numel(), _stream(b),
        )
        _lib.check(st, "angle_scan backward")
        return dtheta, dscale, dgamma, db, dh0


@_angle_scan_bwd.register_fake
def _(theta, scale, gamma, b, h0, perm, sgn, p2p, h, grad_h, carries, has_scale, has_decay, brickwall):
    return (torch.empty_like(theta), torch.empty_like(scale), torch.empty_like(gamma),
            torch.empty_like(b), torch.empty_like(h0))


def _angle_setup(ctx, inputs, output):
    theta, scale, gamma, b, h0, perm, sgn, p2p, has_scale, has_decay, brickwall, _ = inputs
    h, carries = output
    ctx.save_for_backward(theta, scale, gamma, b, h0, perm, sgn, p2p, h, carries)
    ctx.flags = (has_scale, has_decay, brickwall)
    ctx.mark_non_differentiable(carries)
    ctx.set_materialize_grads(False)


def _angle_backward(ctx, grad_h, _gcarries):
    if torch.is_grad_enabled():
        raise RuntimeError("angle_scan does not support second-order autograd (create_graph=True)")
    if grad_h is None:
        return (None,) * 12
    theta, scale, gamma, b, h0, perm, sgn, p2p, h, carries = ctx.saved_tensors
    has_scale, has_decay, brickwall = ctx.flags
    dth, dsc, dga, db, dh0 = _angle_scan_bwd(
        theta, scale, gamma, b, h0, perm, sgn, p2p, h, grad_h, carries, has_scale, has_decay,
        brickwall,
    )
    return dth, dsc, dga, db, dh0, None, None, None, None, None, None, None


torch.library.register_autograd(
    "mingru_b200::angle_scan_fwd", _angle_backward, setup_context=_angle_setup
)


def angle_scan_impl(
    theta: torch.Tensor, scale: torch.Tensor, gamma: torch.Tensor, b: torch.Tensor,
    h0: torch.Tensor, perm: torch.Tensor, sgn: torch.Tensor, p2p: torch.Tensor,
    *, has_scale: int, has_decay: int,
) -> torch.Tensor:
    """Angle-fused Givens / rotation scan; returns the states ``h`` ``(B, T, n, k)``.

    Same arguments and contract as the reference's
    ``triton_scans.angle_scan_impl`` (``triton_scans.py:1743-1812``):
    ``theta`` ``(B, T, n, R, k/2)``, ``scale`` / ``gamma`` ``(B, T, n)``
    (read only when ``has_scale`` / ``has_decay``), ``b`` ``(B, T, n, k)``,
    ``h0`` ``(B, n, k)``, plane metadata ``perm`` / ``sgn`` / ``p2p`` ``(R, k)``.
    Differentiable w.r.t. theta, scale, gamma, b and h0.
    """
    op = "angle_scan"
    if theta.ndim != 5 or b.ndim != 4:
        raise ValueError(
            f"{op}: need 5-D (B, T, n, R, half) theta and 4-D (B, T, n, k) b "
            f"(got theta={tuple(theta.shape)}, b={tuple(b.shape)})"
        )
    Bn, T, n, R, half = theta.shape
    k = b.shape[-1]
    if (k < 2 or k % 2 or 2 * half != k or b.shape[:3] != (Bn, T, n)
            or tuple(scale.shape) != (Bn, T, n) or tuple(gamma.shape) != (Bn, T, n)
            or tuple(h0.shape) != (Bn, n, k) or tuple(perm.shape) != (R, k)
            or tuple(sgn.shape) != (R, k) or tuple(p2p.shape) != (R, k)):
        raise ValueError(
            f"{op}: shapes disagree (theta={tuple(theta.shape)}, scale={tuple(scale.shape)}, "
            f"gamma={tuple(gamma.shape)}, b={tuple(b.shape)}, h0={tuple(h0.shape)}, "
            f"perm={tuple(perm.shape)}): need an even k = 2 * half and scale/gamma/b/h0/"
            "perm/sgn/p2p agreeing with theta's (B, T, n, R, half) on (B, T, n, R, k)"
        )
    if k > 64 or R > 16:
        raise ValueError(f"{op}: k <= 64 and R <= 16 supported (got k={k}, R={R})")
    _require_cuda(op, theta, scale, gamma, b, h0, perm, sgn, p2p)
    dt = b.dtype
    if any(x.dtype != dt for x in (theta, scale, gamma, h0)):
        raise ValueError(f"{op}: theta, scale, gamma, b and h0 must share a dtype")
    _dtype_code(op, b)
    perm = perm.to(torch.int32).contiguous()
    p2p = p2p.to(torch.int32).contiguous()
    sgn = sgn.to(torch.float32).contiguous()
    brick = 1 if _is_brickwall(perm, sgn, p2p) else 0
    need = torch.is_grad_enabled() and any(
        x.requires_grad for x in (theta, scale, gamma, b, h0))
    h, _ = _angle_scan_fwd(theta, scale, gamma, b, h0, perm, sgn, p2p,
                           int(has_scale), int(has_decay), brick, need)
    return h


# ================================================ DeltaMinGRU chunked-WY ==


def _delta_dims(Q, K, V):
    Bn, H, T, dk = Q.shape
    return Bn, H, T, K.shape[3], dk, V.shape[4]


@torch.library.custom_op("mingru_b200::delta_fwd", mutates_args=())
def _delta_fwd(
    Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, beta: torch.Tensor, H0: torch.Tensor,
    chunk_size: int,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(Q.device):  # sizes are queried on the launch device
        Q, K, V, beta = (_dense(x) for x in (Q, K, V, beta))
        H0 = _dense(H0.float())
        Bn, H, T, nh, dk, dv = _delta_dims(Q, K, V)
        code = _dtype_code("delta_scan", Q)
        y = torch.empty(Bn, H, T, dv, dtype=Q.dtype, device=Q.device)
        HT = torch.empty(Bn, H, dk, dv, dtype=torch.float32, device=Q.device)
        saved = torch.empty(lib.mgs_delta_saved_size(Bn, H, T, nh, dk, dv, chunk_size, code) // 4,
                            dtype=torch.float32, device=Q.device)
        ws = _workspace(lib.mgs_delta_workspace_size(Bn, H, T, nh, dk, dv, chunk_size, code), Q.device)
        st = lib.mgs_delta_fwd(
            _ptr(Q), _ptr(K), _ptr(V), _ptr(beta), _ptr(H0), _ptr(y), _ptr(HT), _ptr(saved),
            Bn, H, T, nh, dk, dv, chunk_size, code, _ptr(ws), ws.numel(), _stream(Q),
        )
        _lib.check(st, "delta_scan forward")
        return y, HT, saved


@_delta_fwd.register_fake
def _(Q, K, V, beta, H0, chunk_size):
    Bn, H, T, nh, dk, dv = _delta_dims(Q, K, V)
    n = _lib.load().mgs_delta_saved_size(Bn, H, T, nh, dk, dv, chunk_size,
                                         _dtype_code("delta_scan", Q)) // 4
    return (Q.new_empty((Bn, H, T, dv)), Q.new_empty((Bn, H, dk, dv), dtype=torch.float32),
            Q.new_empty((n,), dtype=torch.float32))


@torch.library.custom_op("mingru_b200::delta_bwd", mutates_args=())
def _delta_bwd(
    Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, beta: torch.Tensor, saved: torch.Tensor,
    dy: torch.Tensor, dHT: torch.Tensor, chunk_size: int,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(Q.device):  # sizes are queried on the launch device
        Q, K, V, beta = (_dense(x) for x in (Q, K, V, beta))
        dy = _dense(dy.to(Q.dtype))
        dHT = _dense(dHT.float())
        Bn, H, T, nh, dk, dv = _delta_dims(Q, K, V)
        code = _dtype_code("delta_scan", Q)
        dQ, dK, dV, db = (torch.empty_like(x) for x in (Q, K, V, beta))
        dH0 = torch.empty(Bn, H, dk, dv, dtype=torch.float32, device=Q.device)
        ws = _workspace(lib.mgs_delta_workspace_size(Bn, H, T, nh, dk, dv, chunk_size, code), Q.device)
        st = lib.mgs_delta_bwd(
            _ptr(Q), _ptr(K), _ptr(V), _ptr(beta), _ptr(saved), _ptr(dy), _ptr(dHT),
            _ptr(dQ), _ptr(dK), _ptr(dV), _ptr(db), _ptr(dH0),
            Bn, H, T, nh, dk, dv, chunk_size, code, _ptr(ws), ws.numel(), _stream(Q),
        )
        _lib.check(st, "delta_scan backward")
        return dQ, dK, dV, db, dH0


@_delta_bwd.register_fake
def _(Q, K, V, beta, saved, dy, dHT, chunk_size):
    Bn, H, T, nh, dk, dv = _delta_dims(Q, K, V)
    return (torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V), torch.empty_like(beta),
            Q.new_empty((Bn, H, dk, dv), dtype=torch.float32))


def _delta_setup(ctx, inputs, output):
    Q, K, V, beta, H0, chunk_size = inputs
    y, HT, saved = output
    ctx.save_for_backward(Q, K, V, beta, saved)
    ctx.chunk_size = chunk_size
    ctx.h0_dtype = H0.dtype
    ctx.mark_non_differentiable(saved)
    ctx.set_materialize_grads(False)


def _delta_backward(ctx, dy, dHT, _gsaved):
    if torch.is_grad_enabled():
        raise RuntimeError("delta_scan does not support second-order autograd (create_graph=True)")
    Q, K, V, beta, saved = ctx.saved_tensors
    if dy is None and dHT is None:
        return None, None, None, None, None, None
    Bn, H, T, nh, dk, dv = _delta_dims(Q, K, V)
    if dy is None:
        dy = torch.zeros(Bn, H, T, dv, dtype=Q.dtype, device=Q.device)
    if dHT is None:
        dHT = torch.zeros(Bn, H, dk, dv, dtype=torch.float32, device=Q.device)
    dQ, dK, dV, db, dH0 = _delta_bwd(Q, K, V, beta, saved, dy, dHT, ctx.chunk_size)
    return dQ, dK, dV, db, dH0.to(ctx.h0_dtype), None


torch.library.register_autograd("mingru_b200::delta_fwd", _delta_backward, setup_context=_delta_setup)

@torch.library.custom_op("mingru_b200::delta_gated_fwd", mutates_args=())
def _delta_gated_fwd(
    Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, beta: torch.Tensor, H0: torch.Tensor,
    log_gamma: torch.Tensor, chunk_size: int,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(Q.device):  # sizes are queried on the launch device
        Q, K, V, beta = (_dense(x) for x in (Q, K, V, beta))
        H0 = _dense(H0.float())
        lg = _dense(log_gamma.float())
        Bn, H, T, nh, dk, dv = _delta_dims(Q, K, V)
        code = _dtype_code("delta_scan", Q)
        y = torch.empty(Bn, H, T, dv, dtype=Q.dtype, device=Q.device)
        HT = torch.empty(Bn, H, dk, dv, dtype=torch.float32, device=Q.device)
        n = lib.mgs_delta_gated_saved_size(Bn, H, T, nh, dk, dv, chunk_size, code)
        saved = torch.empty(n // 4, dtype=torch.float32, device=Q.device)
        ws = _workspace(lib.mgs_delta_gated_workspace_size(Bn, H, T, nh, dk, dv, chunk_size, code),
                        Q.device)
        st = lib.mgs_delta_gated_fwd(
            _ptr(Q), _ptr(K), _ptr(V), _ptr(beta), _ptr(H0), _ptr(lg), _ptr(y), _ptr(HT),
            _ptr(saved), Bn, H, T, nh, dk, dv, chunk_size, code, _ptr(ws), ws.numel(), _stream(Q),
        )
        _lib.check(st, "delta_scan (decay) forward")
        return y, HT, saved


@_delta_gated_fwd.register_fake
def _(Q, K, V, beta, H0, log_gamma, chunk_size):
    Bn, H, T, nh, dk, dv = _delta_dims(Q, K, V)
    n = _lib.load().mgs_delta_gated_saved_size(Bn, H, T, nh, dk, dv, chunk_size,
                                               _dtype_code("delta_scan", Q)) // 4
    return (Q.new_empty((Bn, H, T, dv)), Q.new_empty((Bn, H, dk, dv), dtype=torch.float32),
            Q.new_empty((n,), dtype=torch.float32))


@torch.library.custom_op("mingru_b200::delta_gated_bwd", mutates_args=())
def _delta_gated_bwd(
    Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, beta: torch.Tensor, log_gamma: torch.Tensor,
    saved: torch.Tensor, dy: torch.Tensor, dHT: torch.Tensor, chunk_size: int,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    with torch.cuda.device(Q.device):  # sizes are queried on the launch device
        Q, K, V, beta = (_dense(x) for x in (Q, K, V, beta))
        lg = _dense(log_gamma.float())
        dy = _dense(dy.to(Q.dtype))
        dHT = _dense(dHT.float())
        Bn, H, T, nh, dk, dv = _delta_dims(Q, K, V)
        code = _dtype_code("delta_scan", Q)
        dQ, dK, dV, db = (torch.empty_like(x) for x in (Q, K, V, beta))
        dH0 = torch.empty(Bn, H, dk, dv, dtype=torch.float32, device=Q.device)
        dlg = torch.empty(Bn, H, T, dtype=torch.float32, device=Q.device)
        ws = _workspace(lib.mgs_delta_gated_workspace_size(Bn, H, T, nh, dk, dv, chunk_size, code),
                        Q.device)
        st = lib.mgs_delta_gated_bwd(
            _ptr(Q), _ptr(K), _ptr(V), _ptr(beta), _ptr(lg), _ptr(saved), _ptr(dy), _ptr(dHT),
            _ptr(dQ), _ptr(dK), _ptr(dV), _ptr(db), _ptr(dH0), _ptr(dlg),
            Bn, H, T, nh, dk, dv, chunk_size, code, _ptr(ws), ws.numel(), _stream(Q),
        )
        _lib.check(st, "delta_scan (decay) backward")
        return dQ, dK, dV, db, dH0, dlg


@_delta_gated_bwd.register_fake
def _(Q, K, V, beta, log_gamma, saved, dy, dHT, chunk_size):
    Bn, H, T, nh, dk, dv = _delta_dims(Q, K, V)
    return (torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V), torch.empty_like(beta),
            Q.new_empty((Bn, H, dk, dv), dtype=torch.float32),
            Q.new_empty((Bn, H, T), dtype=torch.float32))


def _delta_gated_setup(ctx, inputs, output):
    Q, K, V, beta, H0, lg, chunk_size = inputs
    ctx.save_for_backward(Q, K, V, beta, lg, output[2])
    ctx.chunk_size = chunk_size
    ctx.h0_dtype = H0.dtype
    ctx.lg_dtype = lg.dtype
    ctx.mark_non_differentiable(output[2])
    ctx.set_materialize_grads(False)


def _delta_gated_backward(ctx, dy, dHT, _gsaved):
    if torch.is_grad_enabled():
        raise RuntimeError("delta_scan does not support second-order autograd (create_graph=True)")
    Q, K, V, beta, lg, saved = ctx.saved_tensors
    if dy is None and dHT is None:
        return (None,) * 7
    Bn, H, T, nh, dk, dv = _delta_dims(Q, K, V)
    if dy is None:
        dy = torch.zeros(Bn, H, T, dv, dtype=Q.dtype, device=Q.device)
    if dHT is None:
        dHT = torch.zeros(Bn, H, dk, dv, dtype=torch.float32, device=Q.device)
    dQ, dK, dV, db, dH0, dlg = _delta_gated_bwd(Q, K, V, beta, lg, saved, dy, dHT, ctx.chunk_size)
    return dQ, dK, dV, db, dH0.to(ctx.h0_dtype), dlg.to(ctx.lg_dtype), None


torch.library.register_autograd(
    "mingru_b200::delta_gated_fwd", _delta_gated_backward, setup_context=_delta_gated_setup
)


def delta_gated_scan_impl(
    Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, beta: torch.Tensor, H0: torch.Tensor,
    log_gamma: torch.Tensor, *, chunk_size: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    """The delta rule with per-token time decay; returns ``(y, H_T)``.

    Arguments as :func:`delta_scan_impl`, plus ``log_gamma`` ``(B, n_heads, T)``
    (or broadcastable to it): the per-token log decay ``-lambda * dt <= 0`` of
    each head. The state entering token t decays by ``exp(log_gamma_t)``
    before the token's ``nh`` micro-steps -- the decay-active
    ``DeltaMinGRU._forward_chunked_gated`` (reference ``min_gru.py:3290-3448``),
    which the reference runs in eager torch only. Every decay factor is exp of
    a chunk-relative span sum (no division, no difference of running sums), so
    a saturated gap wipes the memory exactly. Differentiable w.r.t. all six
    tensors (``log_gamma`` included, so lambda and dt get gradients through it).
    """
    op = "delta_scan"
    if Q.ndim != 4:
        raise ValueError(f"{op}: need 4-D Q (B, n_heads, T, d_k) (got {tuple(Q.shape)})")
    Bn, H, T, dk = Q.shape
    lg = torch.broadcast_to(log_gamma, (Bn, H, T))
    return _delta_checked(Q, K, V, beta, H0, chunk_size, gated=True, log_gamma=lg)


_DELTA_MAX_DK = 128
_DELTA_DV_BLOCK = 64  # value columns per kernel call: wider d_v runs as column blocks


def delta_scan_impl(
    Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, beta: torch.Tensor, H0: torch.Tensor,
    *, chunk_size: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    return _delta_checked(Q, K, V, beta, H0, chunk_size)


def _delta_checked(
    Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, beta: torch.Tensor, H0: torch.Tensor,
    chunk_size: int, gated: bool = False, log_gamma: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """DeltaMinGRU chunked-WY delta rule; returns ``(y, H_T)``.

    Same arguments and layout as the reference's
    ``triton_scans.delta_scan_impl`` (``triton_scans.py:2403-2447``): ``Q``
    ``(B, n_heads, T, d_k)``, ``K`` ``(B, n_heads, T, nh, d_k)``, ``V``
    ``(B, n_heads, T, nh, d_v)``, ``beta`` ``(B, n_heads, T, nh)``, ``H0``
    ``(B, n_heads, d_k, d_v)``. ``y`` ``(B, n_heads, T, d_v)`` has the inputs'
    dtype; the state ``H_T`` is fp32 (``H0``'s dtype if that is wider).
    Differentiable w.r.t. all five tensors; fp32, bf16 or fp16 inputs (fp32
    arithmetic). Envelope: ``d_k <= 128``, any ``d_v``, ``nh`` and
    ``chunk_size`` whose one-token chunk fits the kernels' shared memory
    (``nh`` up to 96 at ``d_k = d_v = 64``). The chunked form is exact for any
    chunk length, so the kernels may use shorter chunks than ``chunk_size``
    (whole tokens, at most ``64 / nh`` on the tensor-core kernels that bf16
    and fp32 inputs with ``d_k, d_v <= 64`` take) -- the
    result differs only by rounding. The state's value columns evolve
    independently, so ``d_v > 64`` runs as blocks of 64 columns whose
    gradients w.r.t. Q, K and beta add up (in fp32: 16-bit inputs run those
    blocks on fp32 copies).
    """
    op = "delta_scan"
    if Q.ndim != 4 or K.ndim != 5 or V.ndim != 5 or beta.ndim != 4 or H0.ndim != 4:
        raise ValueError(
            f"{op}: need 4-D Q (B, n_heads, T, d_k), 5-D K (B, n_heads, T, nh, d_k), 5-D V "
            "(B, n_heads, T, nh, d_v), 4-D beta (B, n_heads, T, nh) and 4-D H0 (B, n_heads, d_k, "
            f"d_v); got ranks Q={Q.ndim}, K={K.ndim}, V={V.ndim}, beta={beta.ndim}, H0={H0.ndim}"
        )
    Bn, H, T, dk = Q.shape
    nh, dv = K.shape[3], V.shape[4]
    if (K.shape[:3] != (Bn, H, T) or K.shape[4] != dk or V.shape[:3] != (Bn, H, T)
            or V.shape[3] != nh or tuple(beta.shape) != (Bn, H, T, nh)
            or tuple(H0.shape) != (Bn, H, dk, dv)):
        raise ValueError(
            f"{op}: shapes disagree: from Q={tuple(Q.shape)} expected K={(Bn, H, T, nh, dk)}, "
            f"V={(Bn, H, T, nh, dv)}, beta={(Bn, H, T, nh)}, H0={(Bn, H, dk, dv)}; got "
            f"K={tuple(K.shape)}, V={tuple(V.shape)}, beta={tuple(beta.shape)}, H0={tuple(H0.shape)}"
        )
    if chunk_size < 1 or dk > _DELTA_MAX_DK:
        raise ValueError(
            f"{op}: outside the kernel envelope: need chunk_size >= 1 and d_k <= {_DELTA_MAX_DK} "
            f"(got nh={nh}, chunk_size={chunk_size}, d_k={dk}, d_v={dv})"
        )
    _require_cuda(op, Q, K, V, beta, H0)
    if any(x.dtype != Q.dtype for x in (K, V, beta)):
        raise ValueError(f"{op}: Q, K, V and beta must share a dtype")
    code = _dtype_code(op, Q)
    lib = _lib.load()
    size_fn = lib.mgs_delta_gated_saved_size if gated else lib.mgs_delta_saved_size
    if size_fn(Bn, H, T, nh, dk, min(dv, _DELTA_DV_BLOCK), int(chunk_size), code) == 0 \
            and Bn * H * T > 0:
        raise ValueError(
            f"{op}: outside the kernel envelope: nh={nh} micro-steps of one token do not fit the "
            f"kernels' shared memory at d_k={dk} (chunk_size={chunk_size}, d_v={dv})"
        )
    if gated:
        _require_cuda(op, log_gamma)
        fwd = lambda q, k, v, b, h0: _delta_gated_fwd(q, k, v, b, h0, log_gamma, int(chunk_size))
    else:
        fwd = lambda q, k, v, b, h0: _delta_fwd(q, k, v, b, h0, int(chunk_size))
    if Q.dtype == torch.float16 or (gated and Q.dtype != torch.float32):
        # fp16 inputs, and 16-bit inputs with decay, take the fp32 kernels
        # (tensor cores where the shape allows): fp32 arithmetic either way,
        # rounded once to the input dtype on output.
        y, HT = _delta_checked(Q.float(), K.float(), V.float(), beta.float(), H0, chunk_size,
                               gated, log_gamma)
        return y.to(Q.dtype), HT
    if dv <= _DELTA_DV_BLOCK:
        y, HT, _ = fwd(Q, K, V, beta, H0)
    else:
        # Independent value-column blocks; autograd adds their Q, K, beta
        # gradients. Blocks of 16-bit inputs run in fp32 so the partial
        # gradients are summed before the one rounding to the input dtype.
        wide = (lambda t: t.float()) if Q.dtype != torch.float32 else (lambda t: t)
        Qw, Kw, bw = wide(Q), wide(K), wide(beta)
        ys, hts = [], []
        for j0 in range(0, dv, _DELTA_DV_BLOCK):
            j1 = min(dv, j0 + _DELTA_DV_BLOCK)
            yj, hj, _ = fwd(Qw, Kw, wide(V[..., j0:j1]), bw, H0[..., j0:j1])
            ys.append(yj)
            hts.append(hj)
        y, HT = torch.cat(ys, -1).to(Q.dtype), torch.cat(hts, -1)
    if H0.dtype == torch.float64:
        HT = HT.double()
    return y, HT
