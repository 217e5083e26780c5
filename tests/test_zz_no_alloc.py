"""vmscan_bwd_noalloc: the VJP entry point for callers that cannot allocate device
memory (e.g. a C/FFI binding handed only raw buffers, or a serving process that
forbids allocator calls after start-up).  Its scratch is a static device array
of the library, so this file checks it against the workspace-taking vmscan_bwd
on the same inputs, twice in a row (the array keeps the previous call's
contents), and checks that oversized problems are refused before any launch.
Kept in a file that is collected last so an earlier failure is reported first.
"""

import ctypes

import pytest
import torch

from mlx_vision_mamba_b200 import _native, directions_for
from oracle import scan_ref
from parity import assert_parity

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


@pytest.mark.gpu
@pytest.mark.parametrize("direction", [None, "col"])
def test_noalloc_matches_workspace_entry_point_twice(direction):
    lib = _native.load()
    b, l, dn = 3, 196, 96
    d = directions_for(4, (14, 14))[3] if direction == "col" else None
    dptr = ctypes.byref(d.to_native()) if d is not None else None
    t = _bufs(b, l, dn, seed=21)
    n_ck = lib.vmscan_ckpt_elems(b, l, dn, 16, dptr)
    ck = torch.empty(n_ck, device="cuda")
    y = torch.empty_like(t["u"])
    st = lib.vmscan_fwd(b, l, dn, 16, t["u"].data_ptr(), S(t["u"]), t["delta"].data_ptr(), S(t["delta"]),
                        t["A"].data_ptr(), t["B"].data_ptr(), S(t["B"]), t["C"].data_ptr(), S(t["C"]),
                        t["D"].data_ptr(), t["z"].data_ptr(), S(t["z"]), y.data_ptr(), S(y), ck.data_ptr(), dptr,
                        None, 0, _stream())
    assert st == 0, lib.vmscan_last_error()

    # reference: the workspace-taking entry point
    ref = _outs(b, l, dn)
    ws_n = lib.vmscan_bwd_workspace_bytes(b, l, dn, 16, dptr, 0)
    ws = torch.empty(ws_n, dtype=torch.uint8, device="cuda")
    st = lib.vmscan_bwd(*_args(t, ref, ck, dptr), ws.data_ptr(), ws_n, _stream())
    assert st == 0, lib.vmscan_last_error()
    torch.cuda.synchronize()

    for call in range(2):  # the second call starts from the first call's scratch contents
        got = _outs(b, l, dn)
        st = lib.vmscan_bwd_noalloc(*_args(t, got, ck, dptr), _stream())
        assert st == 0, lib.vmscan_last_error()
        torch.cuda.synchronize()
        for k in ref:
            assert_parity(f"noalloc call {call} {k}", got[k].cpu(), ref[k].double().cpu())

    # without checkpoints the forward is rebuilt inside the static scratch too
    got = _outs(b, l, dn)
    st = lib.vmscan_bwd_noalloc(*_args(t, got, None, dptr), _stream())
    assert st == 0, lib.vmscan_last_error()
    torch.cuda.synchronize()
    for k in ref:
        assert_parity(f"noalloc recompute {k}", got[k].cpu(), ref[k].double().cpu())


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
