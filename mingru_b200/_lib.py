"""ctypes binding of ``libmingru_scan.so`` (the C ABI in ``include/mingru_scan.h``).

The library is built in-tree by ``python -m mingru_b200.build``. There is no
fallback: if it is missing or fails to load, every op raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmingru_scan.so"

MGS_OK = 0
STATUS_NAMES = {
    0: "MGS_OK",
    1: "MGS_BAD_SHAPE",
    2: "MGS_BAD_DTYPE",
    3: "MGS_BAD_ALIGNMENT",
    4: "MGS_UNSUPPORTED",
    5: "MGS_LAUNCH_FAILED",
    6: "MGS_LOOKBACK_TIMEOUT",
    7: "MGS_WORKSPACE_TOO_SMALL",
}
_VALUE_ERRORS = {1, 2, 3, 4}

_p, _i64, _sz, _int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_size_t, ctypes.c_int

# name -> (restype, argtypes); mirrors include/mingru_scan.h exactly.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "mgs_version": (_int, []),
    "mgs_status_string": (ctypes.c_char_p, [_int]),
    "mgs_take_device_error": (_int, [_p]),
    "mgs_linear_scan_workspace_size": (_sz, [_i64, _i64, _i64, _int]),
    "mgs_linear_scan_carry_size": (_sz, [_i64, _i64, _i64, _int]),
    "mgs_linear_scan_fwd": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_linear_scan_bwd": (_int, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_linear_scan_fwd_noalloc": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "mgs_scan_carry_workspace_size": (_sz, [_i64, _i64, _i64]),
    "mgs_linear_scan_carry_fwd": (_int, [_p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_linear_scan_carry_bwd": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_linear_scan_fwd_fixup": (
        _int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_linear_scan_bwd_fixup": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_log_scan_carry_fwd": (_int, [_p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_log_scan_carry_bwd": (_int, [_p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_log_scan_fwd_fixup": (
        _int, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_log_scan_bwd_fixup": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_test_lookback_timeout": (
        _int, [_p, _p, _p, _p, _i64, _i64, _i64, _p, _sz, _i64, _p]),
    "mgs_test_mbarrier_timeout": (_int, [_p, _i64, _p]),
    "mgs_log_scan_workspace_size": (_sz, [_i64, _i64, _i64, _int]),
    "mgs_log_scan_carry_size": (_sz, [_i64, _i64, _i64, _int]),
    "mgs_log_scan_fwd": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_log_scan_bwd": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_log_gate_scan_workspace_size": (_sz, [_i64, _i64, _i64, _int]),
    "mgs_log_gate_scan_carry_size": (_sz, [_i64, _i64, _i64, _int]),
    "mgs_log_gate_scan_fwd": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_log_gate_scan_bwd": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p, _sz, _p]),
    "mgs_affine_scan_workspace_size": (_sz, [_i64, _i64, _i64, _int, _int, _int]),
    "mgs_affine_scan_carry_size": (_sz, [_i64, _i64, _i64, _int, _int, _int]),
    "mgs_affine_scan_fwd": (
        _int, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _int, _int, _p, _sz, _p]),
    "mgs_affine_scan_bwd": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _int, _int, _p, _sz, _p]),
    "mgs_angle_scan_workspace_size": (_sz, [_i64, _i64, _i64, _int, _int, _int, _int]),
    "mgs_angle_scan_carry_size": (_sz, [_i64, _i64, _i64, _int, _int, _int, _int]),
    "mgs_angle_scan_fwd": (
        _int,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _int, _int, _int, _int,
         _int, _p, _sz, _p]),
    "mgs_angle_scan_bwd": (
        _int,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int,
         _int, _int, _int, _int, _int, _p, _sz, _p]),
    "mgs_delta_saved_size": (_sz, [_i64, _int, _i64, _int, _int, _int, _int, _int]),
    "mgs_delta_workspace_size": (_sz, [_i64, _int, _i64, _int, _int, _int, _int, _int]),
    "mgs_delta_fwd": (
        _int,
        [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _int, _i64, _int, _int, _int, _int, _int, _p, _sz,
         _p]),
    "mgs_delta_bwd": (
        _int,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _int, _i64, _int, _int, _int, _int,
         _int, _p, _sz, _p]),
    "mgs_delta_gated_saved_size": (_sz, [_i64, _int, _i64, _int, _int, _int, _int, _int]),
    "mgs_delta_gated_workspace_size": (_sz, [_i64, _int, _i64, _int, _int, _int, _int, _int]),
    "mgs_delta_gated_fwd": (
        _int,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _int, _i64, _int, _int, _int, _int, _int, _p,
         _sz, _p]),
    "mgs_delta_gated_bwd": (
        _int,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _int, _i64, _int, _int,
         _int, _int, _int, _p, _sz, _p]),
    "mgs_mingru_step": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _int, _p]),
    "mgs_signed_step": (_int, [_p, _p, _p, _p, _p, _int, _p, _i64, _i64, _int, _p]),
    "mgs_rotation_step": (_int, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _int, _p]),
    "mgs_givens_step": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _int, _int, _int, _p]),
    "mgs_delta_step": (
        _int, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _int, _int, _int, _int, _int, _p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library once (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run `python -m mingru_b200.build` "
                    "(the scan ops have no CPU or eager fallback)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, op: str) -> None:
    """Map an ``mgs_status`` to ValueError (bad input) or RuntimeError (device)."""
    if status == MGS_OK:
        return
    name = STATUS_NAMES.get(status, f"status {status}")
    msg = f"{op}: {name} ({load().mgs_status_string(status).decode()})"
    if status in _VALUE_ERRORS:
        raise ValueError(msg)
    raise RuntimeError(msg)
