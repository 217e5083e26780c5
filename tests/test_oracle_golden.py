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
