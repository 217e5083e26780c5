"""ctypes binding of libvmscan.so (the C ABI declared in include/vmscan.h).

The library is loaded from this package directory.  There is no fallback: if
the library is missing or a CUDA device is not available, the scan entry points
raise.  Build it with ``python -m mlx_vision_mamba_b200.build``.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

LIB_NAME = "libvmscan.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

VMSCAN_OK = 0
VMSCAN_ERR_ALIGN = 4


class Strides(ctypes.Structure):
    """Element strides {batch, seq} of a (batch, seq, channel) view (vmscan_strides)."""

    _fields_ = [("batch", ctypes.c_int64), ("seq", ctypes.c_int64)]


class Direction(ctypes.Structure):
    """Scan direction descriptor (vmscan_direction)."""

    _fields_ = [
        ("ndim", ctypes.c_int32),
        ("grid", ctypes.c_int32 * 4),
        ("axes", ctypes.c_int32 * 4),
        ("reverse", ctypes.c_int32),
    ]


_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t
_S = Strides
_D = ctypes.POINTER(Direction)

# name -> (restype, argtypes); must mirror include/vmscan.h exactly.
SIGNATURES = {
    "vmscan_version": (ctypes.c_int, []),
    "vmscan_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "vmscan_last_error": (ctypes.c_char_p, []),
    "vmscan_ckpt_elems": (_i64, [_i64, _i64, _i64, _i64, _D]),
    "vmscan_fwd_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64, _D]),
    "vmscan_fwd": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i64, _p, _S, _p, _S, _p, _p, _S, _p, _S, _p, _p, _S, _p, _S, _p, _p, _D, _p, _sz, _p],
    ),
    "vmscan_fwd_bf16": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i64, _p, _S, _p, _S, _p, _p, _S, _p, _S, _p, _p, _S, _p, _S, _p, _D, _p, _sz, _p],
    ),
    "vmscan_bwd_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64, _D, ctypes.c_int]),
    "vmscan_bwd": (
        ctypes.c_int,
        [
            _i64, _i64, _i64, _i64,
            _p, _S, _p, _S, _p, _p, _S, _p, _S, _p, _p, _S,  # u delta A B C D z
            _p,  # ckpt
            _p, _S,  # dy
            _p, _S, _p, _S,  # du ddelta
            _p,  # dA
            _p, _S, _p, _S,  # dB dC
            _p,  # dD
            _p, _S, _p,  # dz dz_lo
            _D, _p, _sz, _p,
        ],
    ),
    "vmscan_bwd_bf16": (
        ctypes.c_int,
        [
            _i64, _i64, _i64, _i64,
            _p, _S, _p, _S, _p, _p, _S, _p, _S, _p, _p, _S,  # u delta A B C D z
            _p,  # ckpt
            _p, _S,  # dy
            _p, _S, _p, _S,  # du ddelta
            _p,  # dA
            _p, _S, _p, _S,  # dB dC
            _p,  # dD
            _p, _S,  # dz
            _D, _p, _sz, _p,
        ],
    ),
    "vmscan_bwd_noalloc": (
        ctypes.c_int,
        [
            _i64, _i64, _i64, _i64,
            _p, _S, _p, _S, _p, _p, _S, _p, _S, _p, _p, _S,  # u delta A B C D z
            _p,  # ckpt
            _p, _S,  # dy
            _p, _S, _p, _S,  # du ddelta
            _p,  # dA
            _p, _S, _p, _S,  # dB dC
            _p,  # dD
            _p, _S,  # dz
            _D, _p,
        ],
    ),
    "vmscan_conv1d_silu_fwd": (ctypes.c_int, [_i64, _i64, _i64, _i64, _p, _S, _p, _p, _p, _S, _p, _p, _D, _p]),
    "vmscan_conv1d_bwd_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "vmscan_conv1d_silu_bwd": (
        ctypes.c_int,
        [_i64, _i64, _i64, _i64, _p, _S, _p, _p, _p, _S, _p, _S, _p, _p, _p, _D, _p, _sz, _p],
    ),
    "vmscan_dt_softplus_fwd": (ctypes.c_int, [_i64, _i64, _i64, _p, _i64, _p, _p, _p, _i64, _p]),
    "vmscan_dt_softplus_bwd": (ctypes.c_int, [_i64, _i64, _i64, _p, _i64, _p, _p, _p, _i64, _p, _i64, _p, _p, _p]),
    "vmscan_dt_softplus_bias_rows": (_i64, [_i64]),
    "vmscan_sum_rows": (ctypes.c_int, [_i64, _i64, _p, _p, _p]),
    "vmscan_layernorm_fwd": (ctypes.c_int, [_i64, _i64, _p, _i64, _p, _p, ctypes.c_float, _p, _i64, _p, _p, _p]),
    "vmscan_layernorm_bwd_workspace_bytes": (_i64, [_i64, _i64]),
    "vmscan_layernorm_bwd": (ctypes.c_int, [_i64, _i64, _p, _i64, _p, _p, _p, _p, _i64, _p, _i64, _p, _p, _p,
                                            ctypes.c_size_t, _p]),
    "vmscan_tf32_split": (ctypes.c_int, [_i64, _p, _p, _p, _p]),
    "vmscan_tf32_split_multi": (ctypes.c_int, [ctypes.c_int, _p, _p, _p, _p, _p]),
    "vmscan_gemm_workspace_bytes": (_i64, [_i64, _i64, _i64]),
    "vmscan_gemm_tf32x3": (
        ctypes.c_int,
        [_i64, _i64, _i64, _p, _p, _i64, ctypes.c_int, _p, _p, _i64, ctypes.c_int, _p, _i64, ctypes.c_int, _p, _i64,
         _p],
    ),
    "vmscan_scan_order": (ctypes.c_int, [_i64, _D, ctypes.c_int, _p, _p]),
    "vmscan_device_status": (ctypes.c_int, [_p, ctypes.c_int]),
    "vmscan_wait_timeout_selftest": (ctypes.c_int, [ctypes.c_uint32, _p]),
}

_lib: Optional[ctypes.CDLL] = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libvmscan.so once and declare its signatures.  Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"{LIB_NAME} not found at {path}; build it with `python -m mlx_vision_mamba_b200.build` "
            "(the selective scan has no CPU fallback)"
        )
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _add_nvtx_ranges(lib)
    _lib = lib
    return lib


# Entry points that launch kernels; each call is wrapped in an NVTX range of
# its name so profiler timelines (nsys, ncu --nvtx) group the launches.
TRACED = (
    "vmscan_fwd", "vmscan_bwd", "vmscan_fwd_bf16", "vmscan_bwd_bf16", "vmscan_bwd_noalloc", "vmscan_conv1d_silu_fwd", "vmscan_conv1d_silu_bwd",
    "vmscan_dt_softplus_fwd", "vmscan_dt_softplus_bwd", "vmscan_tf32_split", "vmscan_tf32_split_multi",
    "vmscan_gemm_tf32x3", "vmscan_sum_rows", "vmscan_layernorm_fwd", "vmscan_layernorm_bwd",
)


def _add_nvtx_ranges(lib: ctypes.CDLL) -> None:
    try:
        import torch

        if not torch.cuda.is_available():
            return
        push, pop = torch.cuda.nvtx.range_push, torch.cuda.nvtx.range_pop
    except Exception:  # noqa: BLE001 - tracing is optional
        return

    def traced(name, fn):
        def call(*args):
            push(name)
            try:
                return fn(*args)
            finally:
                pop()

        return call

    for name in TRACED:
        setattr(lib, name, traced(name, getattr(lib, name)))


class VmscanError(RuntimeError):
    """Error status returned by libvmscan.so."""

    def __init__(self, status: int, where: str):
        lib = load()
        msg = lib.vmscan_strerror(int(status)).decode()
        detail = lib.vmscan_last_error().decode()
        super().__init__(f"{where}: vmscan status {status}: {msg}" + (f" ({detail})" if detail else ""))
        self.status = int(status)


def check(status: int, where: str) -> None:
    if status != VMSCAN_OK:
        raise VmscanError(status, where)


def make_direction(ndim: int = 0, grid: Sequence[int] = (), axes: Sequence[int] = (), reverse: bool = False):
    d = Direction()
    d.ndim = int(ndim)
    for i in range(4):
        d.grid[i] = int(grid[i]) if i < len(grid) else 1
        d.axes[i] = int(axes[i]) if i < len(axes) else i
    d.reverse = 1 if reverse else 0
    return d
