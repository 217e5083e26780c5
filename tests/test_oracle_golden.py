"""The CPU oracle against fixtures produced by the reference's own source."""

import pytest
import torch

from conftest import ATOL, RTOL
from golden_cases import MODULE_CASES, SCAN_CASES, build, load, load_params
from oracle import scan_ref


def close(a, b, rtol=RTOL, atol=ATOL):
    torch.testing.assert_close(a, b, rtol=rtol, atol=atol)


@pytest.mark.parametrize("name", SCAN_CASES)
def test_scan_oracle_matches_reference(name):
    rec = load(name)
    y, grads = scan_ref.scan_vjp(rec["inputs"], gated=rec["gated"])
    close(y, rec["y"])
    for k, g in rec["grads"].items():
        close(grads[k], g)


@pytest.mark.parametrize("name", SCAN_CASES)
def test_chunked_oracle_matches_reference(name):
    rec = load(name)
    i = rec["inputs"]
    y = scan_ref.selective_scan_chunked(i["u"], i["delta"], i["A"], i["B"], i["C"], i["D"])
    close(y, rec["y_chunked"])


@pytest.mark.parametrize("name", sorted(MODULE_CASES))
def test_module_oracle_matches_reference(name):
    kind, kw = MODULE_CASES[name]
    rec = load(name)
    mod = build(kind, kw, "oracle")
    load_params(mod, rec["params"])
    x = rec["x"].clone().requires_grad_(True)
    y = mod(x)
    (y * rec["dy"]).sum().backward()
    close(y.detach(), rec["y"])
    close(x.grad, rec["dx"])
    got = dict(mod.named_parameters())
    for k, g in rec["grads"].items():
        gg = got[k].grad if got[k].grad is not None else torch.zeros_like(got[k])
        close(gg.reshape(g.shape), g)


def test_oracle_scan_passes_gradcheck():
    """fp64 gradcheck of the restated sequential scan (with the gate): the
    oracle's autograd gradients are the derivatives of its forward."""
    import torch

    from oracle import scan_ref

    g = torch.Generator().manual_seed(0)
    b, l, d = 1, 5, 3
    u = torch.randn(b, l, d, generator=g, dtype=torch.float64)
    delta = torch.nn.functional.softplus(torch.randn(b, l, d, generator=g, dtype=torch.float64))
    A = -torch.rand(d, 16, generator=g, dtype=torch.float64) - 0.5
    B = torch.randn(b, l, 16, generator=g, dtype=torch.float64)
    C = torch.randn(b, l, 16, generator=g, dtype=torch.float64)
    D = torch.randn(d, generator=g, dtype=torch.float64)
    z = torch.randn(b, l, d, generator=g, dtype=torch.float64)
    args = [t.requires_grad_(True) for t in (u, delta, A, B, C, D, z)]

    def f(u, delta, A, B, C, D, z):
        return scan_ref.selective_scan(u, delta, A, B, C, D) * scan_ref.silu(z)

    assert torch.autograd.gradcheck(f, args, eps=1e-6, atol=1e-7, rtol=1e-6)


def test_chunked_oracle_equals_sequential_in_fp32():
    """The chunked restatement (mamba_fast.py) equals the sequential one."""
    import torch

    from oracle import scan_ref

    inp = scan_ref.sweep_inputs(2, 77, 12, seed=3)
    a = scan_ref.selective_scan(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"])
    c = scan_ref.selective_scan_chunked(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"])
    torch.testing.assert_close(c, a, rtol=1e-6, atol=1e-6)


def test_oracle_in_pieces_equals_one_call():
    """tests/parity.oracle_vjp split over channels or batch rows gives the
    one-call oracle's result (fp64; pieces summed for dB / dC or dA / dD)."""
    from parity import oracle_vjp

    inp = scan_ref.sweep_inputs(3, 20, 40, seed=7)
    y, g = scan_ref.scan_vjp(inp, gated=True, dtype=torch.float64)
    for split, piece in (("channels", 16), ("batch", 2)):
        ys, gs = oracle_vjp(inp, torch.float64, split=split, piece=piece)
        torch.testing.assert_close(ys, y, rtol=1e-13, atol=1e-13)
        assert gs.keys() == g.keys()
        for k in g:
            torch.testing.assert_close(gs[k], g[k], rtol=1e-12, atol=1e-12, msg=f"{split} {k}")
