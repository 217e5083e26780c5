"""LayerNorm over the last dimension on the library's kernels.

The reference normalises the residual blocks' inputs and the encoder's output
with MLX's nn.LayerNorm (mamba_block.py:201,222,401, vision_mamba.py:192: eps
1e-5, affine).  `layer_norm_cuda` runs the forward and the VJP in
`vmscan_layernorm_fwd` / `vmscan_layernorm_bwd` (one warp per row; the weight
and bias gradients summed over rows in a fixed order).  `supported` says which
inputs those kernels take (CUDA fp32, last dimension a multiple of 4 and at
most 1024); `mamba_block.LayerNorm` sends every other input to PyTorch's
layer_norm.
"""

from __future__ import annotations

import torch

from . import _native
from .scan import _ptr, _stream

MAX_DIM = 1024


def supported(x: torch.Tensor, weight, bias) -> bool:
    dim = x.shape[-1] if x.dim() else 0
    return (x.is_cuda and x.dtype == torch.float32 and weight is not None and bias is not None
            and weight.dtype == torch.float32 and bias.dtype == torch.float32 and weight.dim() == 1
            and weight.shape[0] == dim and 0 < dim <= MAX_DIM and dim % 4 == 0 and x.numel() > 0)


def _rows(t: torch.Tensor, dim: int) -> torch.Tensor:
    """t as (rows, dim) with unit column stride, a row stride that is a
    multiple of 4 and a 16-byte aligned base (copied when it is not)."""
    t2 = t.reshape(-1, dim)
    if t2.stride(1) != 1 or t2.stride(0) % 4 or t2.data_ptr() % 16:
        t2 = t2.contiguous()
    return t2


def _param(p: torch.Tensor) -> torch.Tensor:
    p = p.detach()
    return p if p.is_contiguous() and p.data_ptr() % 16 == 0 else p.contiguous()


class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        lib = _native.load()
        dim = x.shape[-1]
        x2 = _rows(x, dim)
        rows = x2.shape[0]
        w, b = _param(weight), _param(bias)
        y = torch.empty((rows, dim), dtype=torch.float32, device=x.device)
        mean = torch.empty((rows,), dtype=torch.float32, device=x.device)
        rstd = torch.empty((rows,), dtype=torch.float32, device=x.device)
        _native.check(lib.vmscan_layernorm_fwd(rows, dim, _ptr(x2), x2.stride(0), _ptr(w), _ptr(b), float(eps),
                                               _ptr(y), y.stride(0), _ptr(mean), _ptr(rstd), _stream(x2)),
                      "vmscan_layernorm_fwd")
        ctx.save_for_backward(x2, w, mean, rstd)
        ctx.x_shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        lib = _native.load()
        x2, w, mean, rstd = ctx.saved_tensors
        rows, dim = x2.shape
        g = _rows(dy, dim)
        dx = torch.empty((rows, dim), dtype=torch.float32, device=x2.device)
        dw = torch.empty((dim,), dtype=torch.float32, device=x2.device)
        db = torch.empty((dim,), dtype=torch.float32, device=x2.device)
        n_ws = lib.vmscan_layernorm_bwd_workspace_bytes(rows, dim)
        if n_ws < 0:
            _native.check(-n_ws, "vmscan_layernorm_bwd_workspace_bytes")
        ws = torch.empty(int(n_ws), dtype=torch.uint8, device=x2.device)
        _native.check(lib.vmscan_layernorm_bwd(rows, dim, _ptr(x2), x2.stride(0), _ptr(w), _ptr(mean), _ptr(rstd),
                                               _ptr(g), g.stride(0), _ptr(dx), dx.stride(0), _ptr(dw), _ptr(db),
                                               _ptr(ws), ws.numel(), _stream(x2)),
                      "vmscan_layernorm_bwd")
        return dx.view(ctx.x_shape), dw, db, None


def layer_norm_cuda(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """LayerNorm of x over its last dimension with the library's kernels
    (inputs for which `supported` holds)."""
    return _LayerNormFn.apply(x, weight, bias, eps)
