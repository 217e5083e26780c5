"""Direction-aware causal depthwise conv1d + SiLU (CUDA) against the reference's
permute -> conv1d -> trim -> silu -> unpermute, restated on the CPU."""

import pytest
import torch
import torch.nn.functional as F

from mlx_vision_mamba_b200 import conv1d_silu_cuda, directions_for
from parity import assert_parity

pytestmark = pytest.mark.gpu


def conv_oracle(x, w, b, direction, dtype):
    """mamba_block.py:129-132,170-171 on the permuted sequence, un-permuted."""
    x = x.to(dtype).clone().requires_grad_(True)
    w = w.to(dtype).clone().requires_grad_(True)
    b = b.to(dtype).clone().requires_grad_(True)
    L, C, K = x.shape[1], x.shape[2], w.shape[1]
    idx = torch.tensor(direction.scan_order(L)) if direction is not None else torch.arange(L)
    inv = torch.empty_like(idx)
    inv[idx] = torch.arange(L)
    xp = x[:, idx]
    y = F.conv1d(xp.transpose(1, 2), w.permute(0, 2, 1), b, padding=K - 1, groups=C).transpose(1, 2)[:, :L]
    y = y * torch.sigmoid(y)
    return y[:, inv], (x, w, b)


def run(b, L, C, K, direction, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(b, L, C, generator=g)
    w = torch.randn(C, K, 1, generator=g) * 0.5
    bias = torch.randn(C, generator=g) * 0.1
    dy = torch.randn(b, L, C, generator=g)
    xc, wc, bc = (t.cuda().requires_grad_(True) for t in (x, w, bias))
    y = conv1d_silu_cuda(xc, wc, bc, direction)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    res = {}
    for dt in (torch.float64, torch.float32):
        yo, leaves = conv_oracle(x, w, bias, direction, dt)
        yo.backward(dy.to(dt))
        res[dt] = (yo.detach(), [lv.grad for lv in leaves])
    (y64, g64), (y32, g32) = res[torch.float64], res[torch.float32]
    tag = f"conv b{b} L{L} C{C} K{K} {direction}"
    assert_parity(tag + " y", y.detach().cpu(), y64, y32)
    for name, got, r64, r32 in zip(("dx", "dw", "db"), (xc.grad, wc.grad, bc.grad), g64, g32):
        assert_parity(f"{tag} {name}", got.cpu(), r64, r32)


@pytest.mark.parametrize("b,L,C,K", [(1, 1, 4, 4), (2, 5, 8, 4), (2, 33, 16, 4), (3, 100, 132, 4), (2, 196, 768, 4),
                                     (1, 40, 12, 2), (1, 70, 8, 7)])
def test_conv_plain(b, L, C, K):
    run(b, L, C, K, None, seed=L + C + K)


@pytest.mark.parametrize("K,grid", [(2, None), (4, (14, 14)), (6, (4, 3, 5)), (8, (2, 3, 2, 4))])
def test_conv_directions(K, grid):
    L = 1
    for gd in grid or (29,):
        L *= gd
    for k, d in enumerate(directions_for(K, grid)):
        run(2, L, 16, 4, d, seed=100 * K + k)


@pytest.mark.parametrize("direction", [None, 1])
def test_conv_full_grid(direction):
    """VisionMamba-2D's batch-64 block shape (1344 CTAs, dw/dbias partials of
    448 (batch, chunk) rows), row-major and column-major scan order."""
    d = directions_for(4, (14, 14))[direction] if direction is not None else None
    run(64, 196, 768, 4, d, seed=7 + (direction or 0))
