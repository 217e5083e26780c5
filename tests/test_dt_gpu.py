"""dt_proj + bias + softplus (CUDA) against the reference's
`log(1 + exp(dt_proj(dt)))` (mlx_vision_mamba/mamba_block.py:177-181),
restated with torch on the CPU in fp64 (exact) and fp32 (the reference's own
precision), values and all three gradients."""

import pytest
import torch

from mlx_vision_mamba_b200 import dt_softplus_cuda
from parity import assert_parity

pytestmark = pytest.mark.gpu


def dt_oracle(x, w, b, dy, dtype):
    x, w, b = (t.to(dtype).clone().requires_grad_(True) for t in (x, w, b))
    y = torch.log(1.0 + torch.exp(x @ w.t() + b))
    y.backward(dy.to(dtype))
    return y.detach(), x.grad, w.grad, b.grad


@pytest.mark.parametrize(
    "b,l,r,dn,wide,scale",
    [
        (2, 196, 24, 768, 56, 1.0),   # VisionMamba: d_model 384 -> dt_rank 24, x_dbc width 24 + 32
        (64, 196, 24, 768, 56, 1.0),  # its batch-64 training shape: 196 dbias partial rows
        (1, 196, 48, 1536, 80, 1.0),  # the published MambaBlock shape: d_model 768 -> dt_rank 48
        (3, 37, 5, 10, 5, 1.0),       # ragged: odd rank, channels off every tile, dense rows
        (1, 64, 64, 300, 64, 3.0),    # largest rank, pre-activations far into both tails
        (1, 1, 16, 4, 16, 1.0),       # single token
    ],
)
def test_dt_softplus_matches_reference(b, l, r, dn, wide, scale):
    g = torch.Generator().manual_seed(r * 1000 + dn)
    xw = torch.randn(b, l, wide, generator=g)
    x = xw[:, :, :r]  # a column slice like x_dbc[..., :dt_rank]
    w = torch.randn(dn, r, generator=g) * scale / r**0.5
    bias = torch.randn(dn, generator=g) * scale
    dy = torch.randn(b, l, dn, generator=g)
    xc = xw.cuda()[:, :, :r].requires_grad_(True)
    wc, bc = w.cuda().requires_grad_(True), bias.cuda().requires_grad_(True)
    y = dt_softplus_cuda(xc, wc, bc)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    y64, dx64, dw64, db64 = dt_oracle(x, w, bias, dy, torch.float64)
    y32, dx32, dw32, db32 = dt_oracle(x, w, bias, dy, torch.float32)
    assert_parity("delta", y.cpu(), y64, y32)
    assert_parity("dx", xc.grad.cpu(), dx64, dx32)
    assert_parity("dweight", wc.grad.cpu(), dw64, dw32)
    assert_parity("dbias", bc.grad.cpu(), db64, db32)


def test_dt_softplus_rejects_bad_rank():
    x = torch.randn(1, 4, 65, device="cuda")
    w = torch.randn(8, 65, device="cuda")
    with pytest.raises(RuntimeError):
        dt_softplus_cuda(x, w, torch.zeros(8, device="cuda"))
