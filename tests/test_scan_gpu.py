"""CUDA selective scan (forward + VJP, gate, directions) against the CPU oracle."""

import ctypes

import pytest
import torch

from golden_cases import SCAN_CASES, load
from mlx_vision_mamba_b200 import BACKWARD, ScanDirection, _native, device_status, directions_for, selective_scan_cuda
from oracle import scan_ref
from parity import assert_parity

pytestmark = pytest.mark.gpu

NAMES = ["u", "delta", "A", "B", "C", "D"]


def cuda_vjp(inp, gated, direction=None, dev="cuda"):
    keys = NAMES + (["z"] if gated else [])
    lv = {k: inp[k].to(dev).float().clone().requires_grad_(True) for k in keys}
    y = selective_scan_cuda(lv["u"], lv["delta"], lv["A"], lv["B"], lv["C"], lv["D"],
                            z=lv.get("z"), direction=direction)
    y.backward(inp["dy"].to(dev).float())
    torch.cuda.synchronize()
    return y.detach().cpu(), {"d" + k: lv[k].grad.detach().cpu() for k in keys}


def oracle_vjp(inp, gated, direction=None, dtype=torch.float64):
    """Oracle on the direction-permuted sequence, results returned in token order."""
    if direction is None:
        return scan_ref.scan_vjp(inp, gated, dtype)
    L = inp["u"].shape[1]
    idx = torch.tensor(direction.scan_order(L))
    inv = torch.empty_like(idx)
    inv[idx] = torch.arange(L)
    p = dict(inp)
    for k in ("u", "delta", "B", "C", "z", "dy"):
        p[k] = inp[k][:, idx]
    y, g = scan_ref.scan_vjp(p, gated, dtype)
    y = y[:, inv]
    for k in ("du", "ddelta", "dB", "dC", "dz"):
        if k in g:
            g[k] = g[k][:, inv]
    return y, g


def check_all(inp, gated, direction=None, tag=""):
    y, g = cuda_vjp(inp, gated, direction)
    y64, g64 = oracle_vjp(inp, gated, direction, torch.float64)
    y32, g32 = oracle_vjp(inp, gated, direction, torch.float32)
    assert_parity(f"{tag} y", y, y64, y32)
    for k in g64:
        assert_parity(f"{tag} {k}", g[k], g64[k], g32[k])


SHAPES = [
    (1, 1, 4, True),
    (2, 2, 8, True),
    (1, 15, 12, False),
    (1, 16, 32, True),
    (2, 17, 40, True),
    (2, 31, 36, False),
    (1, 33, 64, True),
    (3, 100, 40, True),
    (2, 196, 768, True),
    (1, 1024, 32, True),
    (1, 4096, 24, False),
]


@pytest.mark.parametrize("b,l,dn,gated", SHAPES)
def test_scan_matches_oracle(b, l, dn, gated):
    inp = scan_ref.sweep_inputs(b, l, dn, seed=l * 7 + dn)
    check_all(inp, gated, tag=f"({b},{l},{dn},{gated})")


def test_scan_random_A_and_large_delta():
    inp = scan_ref.sweep_inputs(2, 77, 48, seed=5)
    g = torch.Generator().manual_seed(9)
    inp["A"] = -torch.exp(torch.randn(48, 16, generator=g))
    inp["delta"] = torch.nn.functional.softplus(torch.randn(2, 77, 48, generator=g))
    inp["D"] = torch.randn(48, generator=g)
    check_all(inp, True, tag="randA")


@pytest.mark.parametrize(
    "K,grid",
    [(2, None), (4, (14, 14)), (4, (3, 5)), (6, (8, 8, 8)), (6, (2, 3, 5)), (8, (8, 4, 4, 4)), (8, (2, 3, 2, 2))],
)
def test_directions_match_permuted_oracle(K, grid):
    L = 1
    for gdim in grid or (45,):
        L *= gdim
    inp = scan_ref.sweep_inputs(2, L, 32, seed=K * 100 + L)
    for k, d in enumerate(directions_for(K, grid)):
        check_all(inp, True, d, tag=f"K{K} dir{k}")


def test_strided_views_match_contiguous():
    """MambaBlock passes slices of xz and x_dbc; the kernels read them in place."""
    b, l, dn, r = 2, 50, 64, 24
    inp = scan_ref.sweep_inputs(b, l, dn, seed=3)
    xz = torch.cat([inp["u"], inp["z"]], dim=-1).cuda()
    xdbc = torch.cat([torch.randn(b, l, r), inp["B"], inp["C"]], dim=-1).cuda()
    u, z = xz[:, :, :dn], xz[:, :, dn:]
    B, C = xdbc[:, :, r:r + 16], xdbc[:, :, r + 16:]
    dev = {k: inp[k].cuda() for k in ("delta", "A", "D")}
    y1 = selective_scan_cuda(u, dev["delta"], dev["A"], B, C, dev["D"], z=z)
    y2 = selective_scan_cuda(u.contiguous(), dev["delta"], dev["A"], B.contiguous(), C.contiguous(), dev["D"],
                             z=z.contiguous())
    torch.testing.assert_close(y1, y2, rtol=0, atol=0)


def test_unaligned_channel_count_is_padded():
    inp = scan_ref.sweep_inputs(2, 21, 10, seed=4)  # 10 channels: strides not multiples of 4
    check_all(inp, True, tag="dn10")


def test_backward_is_deterministic():
    inp = scan_ref.sweep_inputs(2, 300, 96, seed=11)
    y1, g1 = cuda_vjp(inp, True)
    y2, g2 = cuda_vjp(inp, True)
    assert torch.equal(y1, y2)
    for k in g1:
        assert torch.equal(g1[k], g2[k]), k


def test_bwd_without_checkpoints_recomputes_them():
    """vmscan_bwd(ckpt=NULL) rebuilds the checkpoints like the reference VJP."""
    lib = _native.load()
    b, l, dn = 2, 70, 64
    inp = scan_ref.sweep_inputs(b, l, dn, seed=6)
    t = {k: v.cuda().contiguous() for k, v in inp.items()}
    S = lambda x: _native.Strides(x.stride(0), x.stride(1))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def bwd(ckpt):
        outs = {k: torch.empty_like(t["u"]) for k in ("du", "ddelta", "dz")}
        outs["dA"] = torch.empty(dn, 16, device="cuda")
        outs["dB"] = torch.empty(b, l, 16, device="cuda")
        outs["dC"] = torch.empty(b, l, 16, device="cuda")
        outs["dD"] = torch.empty(dn, device="cuda")
        ws_n = lib.vmscan_bwd_workspace_bytes(b, l, dn, 16, None, int(ckpt is None))
        ws = torch.empty(ws_n, dtype=torch.uint8, device="cuda")
        st = lib.vmscan_bwd(
            b, l, dn, 16, t["u"].data_ptr(), S(t["u"]), t["delta"].data_ptr(), S(t["delta"]), t["A"].data_ptr(),
            t["B"].data_ptr(), S(t["B"]), t["C"].data_ptr(), S(t["C"]), t["D"].data_ptr(), t["z"].data_ptr(),
            S(t["z"]), None if ckpt is None else ckpt.data_ptr(), t["dy"].data_ptr(), S(t["dy"]),
            outs["du"].data_ptr(), S(outs["du"]), outs["ddelta"].data_ptr(), S(outs["ddelta"]),
            outs["dA"].data_ptr(), outs["dB"].data_ptr(), S(outs["dB"]), outs["dC"].data_ptr(), S(outs["dC"]),
            outs["dD"].data_ptr(), outs["dz"].data_ptr(), S(outs["dz"]), None, None, ws.data_ptr(), ws_n, stream)
        assert st == 0, lib.vmscan_strerror(st)
        torch.cuda.synchronize()
        return outs

    n_ck = lib.vmscan_ckpt_elems(b, l, dn, 16, None)
    ck = torch.empty(n_ck, device="cuda")
    y = torch.empty_like(t["u"])
    st = lib.vmscan_fwd(b, l, dn, 16, t["u"].data_ptr(), S(t["u"]), t["delta"].data_ptr(), S(t["delta"]),
                        t["A"].data_ptr(), t["B"].data_ptr(), S(t["B"]), t["C"].data_ptr(), S(t["C"]),
                        t["D"].data_ptr(), t["z"].data_ptr(), S(t["z"]), y.data_ptr(), S(y), None, ck.data_ptr(),
                        None, None, 0, stream)
    assert st == 0
    a = bwd(ck)
    r = bwd(None)
    for k in a:
        assert torch.equal(a[k], r[k]), k


@pytest.mark.parametrize("name", SCAN_CASES)
def test_golden_scan_fixtures(name):
    rec = load(name)
    y, g = cuda_vjp(rec["inputs"], rec["gated"])
    y64, g64 = scan_ref.scan_vjp(rec["inputs"], rec["gated"], torch.float64)
    assert_parity(f"{name} y", y, y64, rec["y"])
    for k in rec["grads"]:
        assert_parity(f"{name} {k}", g[k], g64[k], rec["grads"][k])


def test_errors_are_raised_not_hidden():
    inp = scan_ref.sweep_inputs(1, 8, 8, seed=0)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        selective_scan_cuda(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"])
    t = {k: v.cuda() for k, v in inp.items()}
    with pytest.raises(ValueError, match="d_state"):
        selective_scan_cuda(t["u"], t["delta"], t["A"][:, :8], t["B"][..., :8], t["C"][..., :8], t["D"])


@pytest.mark.parametrize("b,l,dn", [(0, 16, 32), (2, 0, 32), (2, 16, 0)])
@pytest.mark.parametrize("gated", [False, True])
def test_empty_inputs_give_empty_outputs_and_zero_grads(b, l, dn, gated):
    g = torch.Generator().manual_seed(0)
    keys = NAMES + (["z"] if gated else [])
    shapes = {"u": (b, l, dn), "delta": (b, l, dn), "A": (dn, 16), "B": (b, l, 16), "C": (b, l, 16),
              "D": (dn,), "z": (b, l, dn)}
    lv = {k: torch.randn(shapes[k], generator=g).cuda().requires_grad_(True) for k in keys}
    y = selective_scan_cuda(lv["u"], lv["delta"], lv["A"], lv["B"], lv["C"], lv["D"], z=lv.get("z"))
    assert tuple(y.shape) == (b, l, dn) and y.dtype == torch.float32
    y.backward(torch.ones_like(y))
    for k in keys:
        assert lv[k].grad is not None and tuple(lv[k].grad.shape) == shapes[k], k
        assert not lv[k].grad.any(), k
    assert device_status() == 0
    # a direction whose grid does not cover the sequence is refused, empty or not
    with pytest.raises(ValueError, match="does not cover"):
        selective_scan_cuda(lv["u"], lv["delta"], lv["A"], lv["B"], lv["C"], lv["D"],
                            direction=ScanDirection(grid=(4, 4), axes=(1, 0)) if l == 0 else
                            ScanDirection(grid=(4, 5), axes=(1, 0)))


def test_device_status_is_clean():
    inp = scan_ref.sweep_inputs(2, 64, 64, seed=1)
    cuda_vjp(inp, True, ScanDirection(reverse=True))
    assert device_status() == 0


CHUNKED = [
    (1, 4096, 256, True, None),                         # 256 boxes over up to 32 chunks
    (2, 1000, 200, True, "reverse"),                    # ragged last box and chunk, reversed order
    (2, 784, 96, True, "colmajor"),                     # 28 x 28 grid, column-major (K=4 direction 1)
    (1, 512, 40, False, None),
]


@pytest.mark.parametrize("b,l,dn,gated,dirname", CHUNKED)
def test_chunked_scan_matches_oracle_and_unchunked(b, l, dn, gated, dirname):
    """Small batch x channel grids run chunked over L (carry pass + carry chain
    + main pass, forward and VJP): results match the oracle, and the forward
    matches the same scan run in one piece (no workspace) to fp32 rounding."""
    lib = _native.load()
    direction = None
    if dirname == "reverse":
        direction = BACKWARD
    elif dirname == "colmajor":
        direction = directions_for(4, (28, 28))[1]
    dptr = ctypes.byref(direction.to_native()) if direction is not None else None
    assert lib.vmscan_fwd_workspace_bytes(b, l, dn, 16, dptr) > 0, "this shape should be chunked"
    inp = scan_ref.sweep_inputs(b, l, dn, seed=l + dn)
    check_all(inp, gated, direction, tag=f"chunked ({b},{l},{dn},{gated},{dirname})")

    # the forward in one piece: raw ABI call without a workspace
    S = lambda x: _native.Strides(x.stride(0), x.stride(1))  # noqa: E731
    t = {k: v.cuda().float().contiguous() for k, v in inp.items()}
    y1 = torch.empty(b, l, dn, device="cuda")
    st = lib.vmscan_fwd(b, l, dn, 16, t["u"].data_ptr(), S(t["u"]), t["delta"].data_ptr(), S(t["delta"]),
                        t["A"].data_ptr(), t["B"].data_ptr(), S(t["B"]), t["C"].data_ptr(), S(t["C"]),
                        t["D"].data_ptr(), t["z"].data_ptr() if gated else None,
                        S(t["z"]) if gated else _native.Strides(0, 0), y1.data_ptr(), S(y1), None, None, dptr,
                        None, 0, torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.vmscan_last_error()
    y2, _ = cuda_vjp(inp, gated, direction)
    torch.testing.assert_close(y2, y1.cpu(), rtol=1e-4, atol=1e-5)


def test_bounded_wait_times_out_reports_and_context_survives():
    """The failure path of the kernels' bounded waits, triggered on purpose: a
    wait on a barrier that nothing arrives on gives up, the sticky status reads
    VMSCAN_ERR_TIMEOUT once, and the context keeps working."""
    lib = _native.load()
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.vmscan_device_status(stream, 1) == 0
    assert lib.vmscan_wait_timeout_selftest(2000, stream) == 0
    assert lib.vmscan_device_status(stream, 1) == 9  # VMSCAN_ERR_TIMEOUT
    assert lib.vmscan_device_status(stream, 1) == 0
    inp = scan_ref.sweep_inputs(1, 40, 24, seed=11)
    check_all(inp, True, tag="after timeout")
    assert lib.vmscan_device_status(stream, 1) == 0


def test_abi_rejects_views_that_break_the_tma_rules():
    """The C ABI reads sequence tensors through TMA: a view whose base is not
    16-byte aligned or whose strides are not whole 16-byte multiples (4 fp32,
    8 bf16 elements) is rejected with VMSCAN_ERR_ALIGN before any launch (the
    Python layer copies such views instead, test_unaligned_channel_count_is_padded)."""
    lib = _native.load()
    b, l, dn = 2, 32, 64
    S = lambda st: _native.Strides(*st)  # noqa: E731
    dev = "cuda"
    A = -torch.arange(1, 17, dtype=torch.float32, device=dev).repeat(dn, 1)
    D = torch.ones(dn, device=dev)
    y = torch.empty(b, l, dn, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    good = torch.randn(b, l, dn, device=dev)
    bc = torch.randn(b, l, 16, device=dev)

    def fwd(u, su, dt=good, sdt=(l * dn, dn)):
        return lib.vmscan_fwd(b, l, dn, 16, u, S(su), dt.data_ptr(), S(sdt), A.data_ptr(), bc.data_ptr(),
                              S((l * 16, 16)), bc.data_ptr(), S((l * 16, 16)), D.data_ptr(), None, S((0, 0)),
                              y.data_ptr(), S((l * dn, dn)), None, None, None, None, 0, stream)

    assert fwd(good.data_ptr(), (l * dn, dn)) == 0
    wide = torch.randn(b, l, dn + 2, device=dev)  # seq stride 66: not a multiple of 4
    assert fwd(wide.data_ptr(), (l * (dn + 2), dn + 2)) == 4
    assert b"u" in lib.vmscan_last_error()
    assert fwd(good.data_ptr() + 4, (l * dn, dn)) == 4  # base one float past a 16-byte boundary
    assert fwd(good.data_ptr(), (l * dn, dn), dt=wide, sdt=(l * (dn + 2), dn + 2)) == 4
    assert b"delta" in lib.vmscan_last_error()
    # bf16: strides must be multiples of 8 elements
    gb = torch.randn(b, l, dn + 4, device=dev).to(torch.bfloat16)  # seq stride 68: multiple of 4, not 8
    gd = torch.randn(b, l, dn, device=dev).to(torch.bfloat16)
    bcb = bc.to(torch.bfloat16)
    yb = torch.empty(b, l, dn, device=dev, dtype=torch.bfloat16)
    rc = lib.vmscan_fwd_bf16(b, l, dn, 16, gb.data_ptr(), S((l * (dn + 4), dn + 4)), gd.data_ptr(), S((l * dn, dn)),
                             A.data_ptr(), bcb.data_ptr(), S((l * 16, 16)), bcb.data_ptr(), S((l * 16, 16)),
                             D.data_ptr(), None, S((0, 0)), yb.data_ptr(), S((l * dn, dn)), None, None, None, 0,
                             stream)
    assert rc == 4
    torch.cuda.synchronize()
    assert device_status() == 0
