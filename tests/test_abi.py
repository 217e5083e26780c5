"""libvmscan.so loads, exports every function of include/vmscan.h, and validates
arguments on the host (no GPU needed: every call here returns before any CUDA
work)."""

import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT
from mlx_vision_mamba_b200 import _native, directions_for
from mlx_vision_mamba_b200.direction import ScanDirection

HEADER = os.path.join(ROOT, "include", "vmscan.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vmscan_[a-z0-9_]+)\s*\(", text)))


def test_library_loads():
    lib = _native.load()
    assert lib.vmscan_version() >= 100


def test_every_header_function_is_exported_and_bound():
    lib = _native.load()
    names = header_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), f"{n} declared in vmscan.h but not exported"
        assert n in _native.SIGNATURES, f"{n} has no ctypes signature"


def test_strerror_covers_codes():
    lib = _native.load()
    for code in range(0, 12):
        assert lib.vmscan_strerror(code) != b"unknown vmscan status"
    assert lib.vmscan_strerror(99) == b"unknown vmscan status"


def _null_call(lib, **over):
    args = dict(batch=2, seqlen=8, d_inner=32, d_state=16, u=16, delta=16, A=16, B=16, C=16, D=16, y=16)
    args.update(over)
    S = _native.Strides(256, 32)
    return lib.vmscan_fwd(
        args["batch"], args["seqlen"], args["d_inner"], args["d_state"],
        args["u"], S, args["delta"], S, args["A"], args["B"], S, args["C"], S, args["D"],
        None, S, args["y"], S, None, None, None, None, 0, None,
    )


def test_fwd_validation_codes():
    lib = _native.load()
    assert _null_call(lib, d_state=8) == 3  # VMSCAN_ERR_DSTATE
    assert _null_call(lib, A=None) == 1  # VMSCAN_ERR_NULL
    assert _null_call(lib, u=None) == 1
    assert _null_call(lib, batch=0) == 2  # VMSCAN_ERR_SHAPE
    assert _null_call(lib, seqlen=-1) == 2


def test_bad_direction_rejected():
    lib = _native.load()
    bad_grid = _native.make_direction(2, (3, 5), (0, 1))  # 15 != 16
    assert lib.vmscan_ckpt_elems(1, 16, 32, 16, ctypes.byref(bad_grid)) == -5
    bad_axes = _native.make_direction(2, (4, 4), (0, 0))
    assert lib.vmscan_ckpt_elems(1, 16, 32, 16, ctypes.byref(bad_axes)) == -5
    assert lib.vmscan_ckpt_elems(1, 16, 32, 8, None) == -3


def test_ckpt_and_workspace_sizes():
    lib = _native.load()
    # 196 tokens in boxes of 16 -> 13 boxes
    assert lib.vmscan_ckpt_elems(2, 196, 768, 16, None) == 2 * 13 * 768 * 16
    d = directions_for(4, (14, 14))[2]  # column-major: boxes of one column (14 steps)
    assert lib.vmscan_ckpt_elems(2, 196, 768, 16, ctypes.byref(d.to_native())) == 2 * 14 * 768 * 16
    w0 = lib.vmscan_bwd_workspace_bytes(2, 196, 768, 16, None, 0)
    w1 = lib.vmscan_bwd_workspace_bytes(2, 196, 768, 16, None, 1)
    assert w0 > 0 and w1 - w0 >= 2 * 13 * 768 * 16 * 4
    assert lib.vmscan_conv1d_bwd_workspace_bytes(2, 196, 768, 4) > 0
    assert lib.vmscan_conv1d_bwd_workspace_bytes(2, 196, 768, 9) == -10


def _order(d, L, mode):
    lib = _native.load()
    out = np.zeros(L, dtype=np.int64)
    geom = np.zeros(16, dtype=np.int64)
    dptr = ctypes.byref(d.to_native()) if d is not None else None
    st = lib.vmscan_scan_order(L, dptr, mode, out.ctypes.data, geom.ctypes.data)
    assert st == 0
    return out.tolist(), geom


@pytest.mark.parametrize(
    "K,grid",
    [(2, None), (4, (14, 14)), (4, (3, 4)), (4, (5, 7)), (6, (8, 8, 8)), (6, (2, 3, 5)), (8, (8, 4, 4, 4)),
     (8, (2, 2, 3, 2)), (8, (3, 1, 5, 2))],
)
def test_kernel_index_maths_matches_direction_order(K, grid):
    """The kernels' box enumeration and position->token maps visit the tokens in the
    order of the reference's permute/flip (restated in ScanDirection.scan_order)."""
    L = int(np.prod(grid)) if grid else 37
    for d in directions_for(K, grid):
        for mode in (0, 1):
            got, _ = _order(d, L, mode)
            assert got == d.scan_order(L)


def test_scan_order_against_reference_permutation_helpers():
    """Cross-check against the oracle's literal restatement of mamba_block.py:244-338."""
    import torch

    from oracle import model_ref

    for K, grid in ((4, (3, 4)), (6, (2, 3, 4)), (8, (2, 3, 2, 2))):
        L = int(np.prod(grid))
        h = torch.arange(L, dtype=torch.float64).reshape(1, L, 1)
        blk = model_ref.MultiDirectionalMambaBlockRef.__new__(model_ref.MultiDirectionalMambaBlockRef)
        for k, d in enumerate(directions_for(K, grid)):
            pair = k // 2
            if K == 4:
                seq = model_ref.permute_2d_col_major(h, grid) if pair == 1 else h
            else:
                seq = model_ref.permute_axes(h, grid, model_ref._AXIS_PERMS[K][pair])
            if k % 2:
                seq = torch.flip(seq, dims=[1])
            expect = seq.reshape(-1).long().tolist()
            got, _ = _order(d, L, 0)
            assert got == expect, (K, grid, k)


def test_plain_sequence_geometry():
    got, geom = _order(None, 196, 0)
    assert got == list(range(196))
    assert geom[11] == 16 and geom[12] == 13  # T, nboxes
    got, _ = _order(ScanDirection(reverse=True), 33, 0)
    assert got == list(range(32, -1, -1))


def test_gemm_host_validation_and_plan():
    """The tensor-core GEMM's host checks and its K-split plan (no CUDA work:
    every call returns before encoding a tensor map)."""
    lib = _native.load()
    P = ctypes.c_void_p
    assert lib.vmscan_gemm_tf32x3(0, 8, 8, P(16), P(16), 8, 0, P(16), P(16), 8, 0, P(16), 8, 0, None, 0, None) == 2
    assert lib.vmscan_gemm_tf32x3(8, 8, 8, P(16), P(16), 8, 0, P(16), P(16), 8, 0, None, 8, 0, None, 0, None) == 1
    assert lib.vmscan_gemm_tf32x3(8, 16, 8, P(16), P(16), 8, 0, P(16), P(16), 8, 0, P(16), 8, 0, None, 0, None) == 2
    assert lib.vmscan_tf32_split(6, P(16), P(16), P(16), None) == 2
    assert lib.vmscan_tf32_split(8, None, P(16), P(16), None) == 1
    assert lib.vmscan_tf32_split(0, None, None, None, None) == 0
    assert lib.vmscan_gemm_workspace_bytes(0, 8, 8) == -2
    # output tiles that fill the GPU: no split, no workspace
    assert lib.vmscan_gemm_workspace_bytes(12544, 6144, 384) == 0
    # out_proj weight gradient of the 2D model: 3 x 24 tiles, split over K
    ws = lib.vmscan_gemm_workspace_bytes(384, 3072, 12544)
    assert ws >= 2 * 384 * 3072 * 4 and ws % 256 == 0
