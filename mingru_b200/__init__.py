"""mingru_b200 -- the mingru scan hot path as hand-written sm_100a CUDA kernels.

A drop-in for the scan family of chris-santiago/minGRU (``mingru`` 0.2.1):
the four public scan functions and the modules that call them run on the
B200 kernels of ``libmingru_scan.so`` through its C ABI
(``include/mingru_scan.h``). There is no Triton, no backend switch and no CPU
fallback: CPU tensors raise.
"""

from .modules import (
    DeltaMinGRU,
    GivensMinGRU,
    MinGRU,
    MinGRUBlock,
    MinGRUStack,
    RotationMinGRU,
    SignedMinGRU,
    g,
    log_g,
)
from .scan_ops import (
    delta_gated_scan_impl,
    delta_scan_impl,
    angle_scan_impl,
    brickwall_meta,
    linear_scan,
    matrix_affine_scan,
    matrix_scan,
    mingru_gate_scan,
    parallel_scan_log,
    raise_device_error,
    take_device_error,
)

__version__ = "0.1.0"

__all__ = [
    "MinGRU",
    "SignedMinGRU",
    "RotationMinGRU",
    "GivensMinGRU",
    "DeltaMinGRU",
    "MinGRUBlock",
    "MinGRUStack",
    "delta_scan_impl",
    "delta_gated_scan_impl",
    "angle_scan_impl",
    "brickwall_meta",
    "linear_scan",
    "matrix_affine_scan",
    "matrix_scan",
    "mingru_gate_scan",
    "parallel_scan_log",
    "raise_device_error",
    "take_device_error",
]
