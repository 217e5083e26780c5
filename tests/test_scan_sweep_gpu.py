"""Parity at every point of the op sweep (batch {8, 64} x L {196, 1024, 4096} x
d_inner {768, 1536}, gated), at the sizes the bench times, through the
public API `selective_scan_cuda(...).backward(dy)`.

The recurrence never crosses channels, and dB / dC only sum over channels of
one (batch row, step), so two slices of each point have an exact fp64 answer
that the CPU oracle computes in seconds:

* 8 channels (both ends of the first and last 128-channel tiles and of the
  middle) over every batch row and every step: y, du, ddelta, dz, dA, dD;
* the last batch row over every channel and every step: y, du, ddelta, dz,
  dB, dC of that row.

The batch-8 points run the L-chunked forward and VJP (carry passes), the
batch-64 points the unchunked kernels, so both paths are checked at the
sizes the op sweep reports.
"""

import pytest
import torch

from mlx_vision_mamba_b200 import selective_scan_cuda
from oracle import scan_ref
from parity import assert_parity, oracle_vjp

pytestmark = pytest.mark.gpu

SWEEP = [(b, l, d) for b in (8, 64) for l in (196, 1024, 4096) for d in (768, 1536)]


def sweep_inputs_cuda(b, l, dn, seed):
    """The sweep's seeded distributions, generated on the device."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    f = dict(device="cuda", dtype=torch.float32)
    return {
        "u": torch.randn(b, l, dn, generator=g, **f),
        "z": torch.randn(b, l, dn, generator=g, **f),
        "delta": torch.nn.functional.softplus(0.5 * torch.randn(b, l, dn, generator=g, **f) - 3.0),
        "A": -torch.arange(1, 17, **f).repeat(dn, 1),
        "B": torch.randn(b, l, 16, generator=g, **f),
        "C": torch.randn(b, l, 16, generator=g, **f),
        "D": torch.ones(dn, **f),
        "dy": torch.randn(b, l, dn, generator=g, **f),
    }


def edge_channels(dn):
    h = dn // 2
    return [0, 1, 127, 128, h - 1, h, dn - 2, dn - 1]


def gpu_vjp(t):
    lv = {k: t[k].clone().requires_grad_(True) for k in ("u", "delta", "A", "B", "C", "D", "z")}
    y = selective_scan_cuda(lv["u"], lv["delta"], lv["A"], lv["B"], lv["C"], lv["D"], z=lv["z"])
    y.backward(t["dy"])
    torch.cuda.synchronize()
    return y.detach(), {"d" + k: v.grad for k, v in lv.items()}


def check_channels(tag, t, y, g, chans):
    idx = torch.tensor(chans, device="cuda")
    sub = {k: t[k].index_select(-1, idx).cpu() for k in ("u", "z", "delta", "dy")}
    sub.update(A=t["A"][idx].cpu(), D=t["D"][idx].cpu(), B=t["B"].cpu(), C=t["C"].cpu())
    y64, g64 = oracle_vjp(sub, torch.float64, split="batch", piece=8)
    y32, g32 = scan_ref.scan_vjp(sub, gated=True, dtype=torch.float32)
    assert_parity(f"{tag} channels y", y.index_select(-1, idx).cpu(), y64, y32)
    for k in ("du", "ddelta", "dz"):
        assert_parity(f"{tag} channels {k}", g[k].index_select(-1, idx).cpu(), g64[k], g32[k])
    # dA / dD sum batch x L terms per element; the oracle's fp32 reduction is
    # pairwise and close to exact, so they are held to the plain 1e-5 / 1e-6
    # bound element by element
    assert_parity(f"{tag} channels dA", g["dA"][idx].cpu(), g64["dA"])
    assert_parity(f"{tag} channels dD", g["dD"][idx].cpu(), g64["dD"])


def check_row(tag, t, y, g, row):
    sub = {k: t[k][row:row + 1].cpu() for k in ("u", "z", "delta", "dy", "B", "C")}
    sub.update(A=t["A"].cpu(), D=t["D"].cpu())
    y64, g64 = oracle_vjp(sub, torch.float64, split="channels", piece=256)
    y32, g32 = scan_ref.scan_vjp(sub, gated=True, dtype=torch.float32)
    assert_parity(f"{tag} row {row} y", y[row:row + 1].cpu(), y64, y32)
    for k in ("du", "ddelta", "dz", "dB", "dC"):
        assert_parity(f"{tag} row {row} {k}", g[k][row:row + 1].cpu(), g64[k], g32[k])


@pytest.mark.parametrize("b,l,dn", SWEEP, ids=[f"b{b}_l{l}_d{d}" for b, l, d in SWEEP])
def test_sweep_point(b, l, dn):
    t = sweep_inputs_cuda(b, l, dn, seed=b * 1000003 + l * 101 + dn)
    y, g = gpu_vjp(t)
    for k, v in [("y", y)] + list(g.items()):
        assert torch.isfinite(v).all(), k
    tag = f"sweep ({b},{l},{dn})"
    check_channels(tag, t, y, g, edge_channels(dn))
    check_row(tag, t, y, g, b - 1)
