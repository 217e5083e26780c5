"""LayerNorm kernels (vmscan_layernorm_fwd / _bwd through norm.layer_norm_cuda)
against PyTorch's layer_norm in fp64 (the exact result) with the fp32 CPU
result as the reference's own rounding, the module path of
mamba_block.LayerNorm, and determinism of the weight / bias gradients."""

import pytest
import torch
import torch.nn.functional as F

from parity import assert_parity

pytestmark = pytest.mark.gpu


def _case(shape, seed):
    g = torch.Generator().manual_seed(seed)
    dim = shape[-1]
    x = torch.randn(*shape, generator=g) * 2.0 + 0.5
    w = 1.0 + 0.1 * torch.randn(dim, generator=g)
    b = 0.1 * torch.randn(dim, generator=g)
    dy = torch.randn(*shape, generator=g)
    return x, w, b, dy


def _reference(x, w, b, dy, dtype):
    xr, wr, br = (t.detach().clone().to(dtype).requires_grad_(True) for t in (x, w, b))
    y = F.layer_norm(xr, (x.shape[-1],), wr, br, 1e-5)
    y.backward(dy.to(dtype))
    return y.detach(), xr.grad, wr.grad, br.grad


@pytest.mark.parametrize("shape", [(2, 196, 384), (64, 196, 384), (3, 5, 8), (7, 32), (4, 1024), (33, 388)])
def test_layer_norm_matches_reference(shape):
    from mlx_vision_mamba_b200.norm import layer_norm_cuda

    x, w, b, dy = _case(shape, seed=sum(shape))
    exact = _reference(x, w, b, dy, torch.float64)
    ref32 = _reference(x, w, b, dy, torch.float32)
    xc, wc, bc = (t.detach().cuda().requires_grad_(True) for t in (x, w, b))
    y = layer_norm_cuda(xc, wc, bc, 1e-5)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    name = f"layernorm {shape}"
    for tag, got, e, r in zip(("y", "dx", "dw", "db"), (y.detach(), xc.grad, wc.grad, bc.grad), exact, ref32):
        assert_parity(f"{name} {tag}", got.cpu(), e, r)


def test_layer_norm_module_and_fallback():
    from mlx_vision_mamba_b200.mamba_block import LayerNorm

    torch.manual_seed(0)
    for dim in (384, 6):  # 6: not a multiple of 4, PyTorch's layer_norm
        m = LayerNorm(dim).cuda()
        with torch.no_grad():
            m.weight.add_(0.1 * torch.randn(dim, device="cuda"))
            m.bias.add_(0.1 * torch.randn(dim, device="cuda"))
        x = torch.randn(4, 10, dim, device="cuda", requires_grad=True)
        y = m(x)
        y.square().sum().backward()
        x64 = x.detach().double().requires_grad_(True)
        y64 = F.layer_norm(x64, (dim,), m.weight.detach().double(), m.bias.detach().double(), m.eps)
        y64.square().sum().backward()
        assert_parity(f"layernorm module dim {dim} y", y.detach().cpu(), y64.detach().cpu())
        assert torch.allclose(x.grad.double().cpu(), x64.grad.cpu(), rtol=1e-4, atol=1e-5)


def test_layer_norm_gradients_are_deterministic():
    from mlx_vision_mamba_b200.norm import layer_norm_cuda

    x, w, b, dy = _case((64, 196, 384), seed=11)
    outs = []
    for _ in range(2):
        xc, wc, bc = (t.detach().cuda().requires_grad_(True) for t in (x, w, b))
        layer_norm_cuda(xc, wc, bc, 1e-5).backward(dy.cuda())
        outs.append((xc.grad.clone(), wc.grad.clone(), bc.grad.clone()))
    for a, c in zip(*outs):
        assert torch.equal(a, c)
