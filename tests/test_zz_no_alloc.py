"""vmscan_bwd_noalloc: the VJP entry point for callers that cannot allocate device
memory (e.g. a C/FFI binding handed only raw buffers, or a serving process that
forbids allocator calls after start-up).  Its scratch is a static device array
of the library that keeps the previous call's contents, so this file first
fills it with another problem's data, then checks that two calls in a row give
exactly (torch.equal) what the workspace-taking vmscan_bwd gives on the same
inputs, with and without checkpoints, for a problem in one piece over L and
one split into L chunks; and that oversized problems are refused before any
launch.
Kept in a file that is collected last so an earlier failure is reported first.
"""

import ctypes

import pytest
import torch

from mlx_vision_mamba_b200 import _native, directions_for
from oracle import scan_ref

S = lambda x: _native.Strides(x.stride(0), x.stride(1))  # noqa: E731


def _bufs(b, l, dn, seed):
    t = {k: v.cuda().contiguous() for k, v in scan_ref.sweep_inputs(b, l, dn, seed=seed).items()}
    return t


def _outs(b, l, dn):
    o = {k: torch.full((b, l, dn), float("nan"), device="cuda") for k in ("du", "ddelta", "dz")}
    o["dA"] = torch.full((dn, 16), float("nan"), device="cuda")
    o["dB"] = torch.full((b, l, 16), float("nan"), device="cuda")
    o["dC"] = torch.full((b, l, 16), float("nan"), device="cuda")
    o["dD"] = torch.full((dn,), float("nan"), device="cuda")
    return o


def _args(t, o, ck, dptr):
    b, l, dn = t["u"].shape
    return [
        b, l, dn, 16, t["u"].data_ptr(), S(t["u"]), t["delta"].data_ptr(), S(t["delta"]), t["A"].data_ptr(),
        t["B"].data_ptr(), S(t["B"]), t["C"].data_ptr(), S(t["C"]), t["D"].data_ptr(), t["z"].data_ptr(),
        S(t["z"]), None if ck is None else ck.data_ptr(), t["dy"].data_ptr(), S(t["dy"]),
        o["du"].data_ptr(), S(o["du"]), o["ddelta"].data_ptr(), S(o["ddelta"]), o["dA"].data_ptr(),
        o["dB"].data_ptr(), S(o["dB"]), o["dC"].data_ptr(), S(o["dC"]), o["dD"].data_ptr(),
        o["dz"].data_ptr(), S(o["dz"]), dptr,
    ]


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _fwd_ckpt(lib, t, dptr):
    b, l, dn = t["u"].shape
    ck = torch.empty(lib.vmscan_ckpt_elems(b, l, dn, 16, dptr), device="cuda")
    y = torch.empty_like(t["u"])
    st = lib.vmscan_fwd(b, l, dn, 16, t["u"].data_ptr(), S(t["u"]), t["delta"].data_ptr(), S(t["delta"]),
                        t["A"].data_ptr(), t["B"].data_ptr(), S(t["B"]), t["C"].data_ptr(), S(t["C"]),
                        t["D"].data_ptr(), t["z"].data_ptr(), S(t["z"]), y.data_ptr(), S(y), None, ck.data_ptr(),
                        dptr, None, 0, _stream())
    assert st == 0, lib.vmscan_last_error()
    return ck


def _with_workspace(lib, t, ck, dptr):
    """The workspace-taking vmscan_bwd on the same inputs: the expected result."""
    b, l, dn = t["u"].shape
    o = _outs(b, l, dn)
    ws_n = lib.vmscan_bwd_workspace_bytes(b, l, dn, 16, dptr, 1 if ck is None else 0)
    ws = torch.empty(ws_n, dtype=torch.uint8, device="cuda")
    args = _args(t, o, ck, dptr)
    args.insert(-1, None)  # vmscan_bwd's dz_lo (NULL: dz itself), which the no-alloc entry point does not take
    st = lib.vmscan_bwd(*args, ws.data_ptr(), ws_n, _stream())
    assert st == 0, lib.vmscan_last_error()
    torch.cuda.synchronize()
    return o


def _noalloc(lib, t, ck, dptr):
    b, l, dn = t["u"].shape
    o = _outs(b, l, dn)
    st = lib.vmscan_bwd_noalloc(*_args(t, o, ck, dptr), _stream())
    assert st == 0, lib.vmscan_last_error()
    torch.cuda.synchronize()
    return o


def _unchunked_workspace_bytes(b, l, dn):
    """vmscan_bwd's workspace when the VJP runs in one piece over L (checkpoints given)."""
    a = lambda x: (x + 255) // 256 * 256  # noqa: E731
    nboxes, ndt = (l + 15) // 16, (dn + 127) // 128
    part = a(b * nboxes * ndt * 16 * 32 * 4)
    return a(a(part + b * dn * 16 * 4) + b * dn * 4)


# (3, 196, 96): one chunk over L; (1, 4096, 96): a single (batch, channel
# tile) pair, so the VJP splits L into chunks and uses the adjoint-carry
# regions of the scratch too.
SHAPES = [(3, 196, 96), (1, 4096, 96)]


@pytest.mark.gpu
@pytest.mark.parametrize("direction", [None, "col"])
@pytest.mark.parametrize("shape", SHAPES)
def test_noalloc_equals_workspace_entry_point(shape, direction):
    lib = _native.load()
    b, l, dn = shape
    if direction == "col" and l != 196:
        pytest.skip("the column-major direction is defined on the 14 x 14 grid")
    d = directions_for(4, (14, 14))[3] if direction == "col" else None
    dptr = ctypes.byref(d.to_native()) if d is not None else None
    if l == 4096:
        assert lib.vmscan_bwd_workspace_bytes(b, l, dn, 16, dptr, 0) > _unchunked_workspace_bytes(b, l, dn)

    # first leave the scratch full of another problem's data: the other
    # shape, with and without checkpoints
    other = SHAPES[1] if shape == SHAPES[0] else SHAPES[0]
    to = _bufs(*other, seed=5)
    _noalloc(lib, to, None, None)
    _noalloc(lib, to, _fwd_ckpt(lib, to, None), None)
    del to

    t = _bufs(b, l, dn, seed=21)
    ck = _fwd_ckpt(lib, t, dptr)
    for ckpt in (ck, None):  # checkpoints given / rebuilt inside the scratch
        ref = _with_workspace(lib, t, ckpt, dptr)
        for call in range(2):  # the second call starts from the first call's scratch contents
            got = _noalloc(lib, t, ckpt, dptr)
            for k in ref:
                assert torch.equal(got[k], ref[k]), (f"noalloc call {call} ckpt={'given' if ckpt is not None else 'NULL'}"
                                                     f" {k}: max diff {(got[k] - ref[k]).abs().max().item():.3e}")


@pytest.mark.gpu
def test_noalloc_refuses_problems_larger_than_its_scratch():
    lib = _native.load()
    b, l, dn = 64, 4096, 1536  # needs ~1.6 GB of scratch
    need = lib.vmscan_bwd_workspace_bytes(b, l, dn, 16, None, 0)
    assert need > 32 * 1024 * 1024
    t = _bufs(1, 8, 16, seed=1)  # any valid device pointers; nothing may be launched
    o = _outs(1, 8, 16)
    args = _args(t, o, None, None)
    args[0:3] = [b, l, dn]
    st = lib.vmscan_bwd_noalloc(*args, _stream())
    assert st == 11, lib.vmscan_strerror(st)
    assert b"static" in lib.vmscan_strerror(st)
    torch.cuda.synchronize()
    assert torch.isnan(o["du"]).all()  # untouched
