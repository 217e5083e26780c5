"""bf16 I/O variant of the CUDA selective scan (vmscan_fwd_bf16 /
vmscan_bwd_bf16): sequence tensors in bf16, A, D, the state and all
arithmetic in fp32.

Two checks per case.  (1) Against the oracle in fp64 on the same
bf16-rounded inputs, with the bf16 rounding of each output added to the fp32
parity bound (tests/parity.py:assert_parity_bf16); dA and dD stay fp32 and
meet the plain fp32 rule.  (2) Against the fp32 kernels on the same rounded
inputs: the bf16 kernels widen every load exactly and run the fp32 kernels'
operations, so each bf16 output equals the fp32 kernels' output rounded to
bf16 (nearest even), and dA, dD are equal bit for bit.
"""

import pytest
import torch

from mlx_vision_mamba_b200 import BACKWARD, directions_for, selective_scan_cuda
from oracle import scan_ref
from parity import assert_parity, assert_parity_bf16

pytestmark = pytest.mark.gpu

SEQ = ("u", "delta", "B", "C", "z", "dy")
NAMES = ["u", "delta", "A", "B", "C", "D"]


def rounded_inputs(b, l, dn, seed):
    inp = scan_ref.sweep_inputs(b, l, dn, seed=seed)
    return {k: (v.to(torch.bfloat16).float() if k in SEQ else v) for k, v in inp.items()}


def run(inp, gated, direction, dtype):
    keys = NAMES + (["z"] if gated else [])
    lv = {}
    for k in keys:
        t = inp[k].cuda()
        lv[k] = (t.to(dtype) if k in SEQ else t.float()).clone().requires_grad_(True)
    y = selective_scan_cuda(lv["u"], lv["delta"], lv["A"], lv["B"], lv["C"], lv["D"], z=lv.get("z"),
                            direction=direction)
    assert y.dtype == dtype
    y.backward(inp["dy"].cuda().to(dtype))
    torch.cuda.synchronize()
    grads = {"d" + k: lv[k].grad.detach().cpu() for k in keys}
    for k in ("du", "ddelta", "dB", "dC", "dz"):
        if k in grads:
            assert grads[k].dtype == dtype, (k, grads[k].dtype)
    return y.detach().cpu(), grads


def oracle(inp, gated, direction, dtype):
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


CASES = [
    (1, 1, 8, True, None),
    (2, 17, 40, True, None),
    (1, 33, 12, False, None),            # channels padded to a whole 16 bytes in storage
    (2, 196, 768, True, None),
    (2, 196, 768, True, "reverse"),
    (2, 196, 192, True, "colmajor"),     # K=4 direction 2 on the 14 x 14 patch grid
    (2, 512, 48, True, "3d"),            # K=6 direction on an 8 x 8 x 8 grid
    (1, 4096, 256, True, None),          # chunked over L (fwd and VJP)
    (2, 1000, 200, True, "reverse"),     # chunked, ragged last box and chunk
]


def _direction(name, l):
    if name is None:
        return None
    if name == "reverse":
        return BACKWARD
    if name == "colmajor":
        return directions_for(4, (14, 14))[2]
    if name == "3d":
        return directions_for(6, (8, 8, 8))[3]
    raise ValueError(name)


@pytest.mark.parametrize("b,l,dn,gated,dirname", CASES)
def test_bf16_scan_matches_oracle_and_fp32_kernels(b, l, dn, gated, dirname):
    direction = _direction(dirname, l)
    inp = rounded_inputs(b, l, dn, seed=l * 3 + dn)
    yb, gb = run(inp, gated, direction, torch.bfloat16)
    tag = f"({b},{l},{dn},{gated},{dirname})"

    y64, g64 = oracle(inp, gated, direction, torch.float64)
    y32, g32 = oracle(inp, gated, direction, torch.float32)
    assert_parity_bf16(f"{tag} y", yb, y64, y32)
    for k in g64:
        if k in ("dA", "dD"):
            assert gb[k].dtype == torch.float32
            assert_parity(f"{tag} {k}", gb[k], g64[k], g32[k])
        else:
            assert_parity_bf16(f"{tag} {k}", gb[k], g64[k], g32[k])

    yf, gf = run(inp, gated, direction, torch.float32)
    assert torch.equal(yb, yf.to(torch.bfloat16)), f"{tag} y differs from bf16(fp32 kernels)"
    for k in gf:
        want = gf[k] if k in ("dA", "dD") else gf[k].to(torch.bfloat16)
        assert torch.equal(gb[k], want), f"{tag} {k} differs from the fp32 kernels' result"


def test_bf16_strided_views_pass_through():
    """x and z as column slices of one bf16 (B, L, 2 D_inner) tensor, like the
    reference's xz split: no copies, same results as contiguous inputs."""
    b, l, dn = 2, 64, 96
    inp = rounded_inputs(b, l, dn, seed=5)
    xz = torch.cat([inp["u"], inp["z"]], dim=-1).cuda().to(torch.bfloat16)
    rest = {k: inp[k].cuda() for k in ("delta", "B", "C")}
    A, D = inp["A"].cuda(), inp["D"].cuda()
    y1 = selective_scan_cuda(xz[:, :, :dn], rest["delta"].bfloat16(), A, rest["B"].bfloat16(), rest["C"].bfloat16(),
                             D, z=xz[:, :, dn:])
    y2 = selective_scan_cuda(xz[:, :, :dn].contiguous(), rest["delta"].bfloat16(), A, rest["B"].bfloat16(),
                             rest["C"].bfloat16(), D, z=xz[:, :, dn:].contiguous())
    assert torch.equal(y1, y2)
