"""fp32 projections on the B200 tensor cores (in_proj / out_proj of the block).

`linear_tc(x, weight)` is `x @ weight.T` (nn.Linear without bias) computed by
libvmscan's tcgen05 GEMM from hi / lo TF32 splits of both operands
(vmscan_tf32_split, vmscan_gemm_tf32x3): three tensor-core products per
output with the large and the correction products in separate fp32
accumulators, accurate to about fp32's own rounding.  The backward pass runs
the same kernel for the input gradient (dy @ weight, weight read MN-major) and
the weight gradient (dy^T @ x, both read MN-major): no transposed copies.

The reference's projections are MLX nn.Linear (mamba_block.py:125,153 and
their calls at :165,191); the direction sum of the multi-directional block
(:562-566) is one out_proj GEMM over the concatenated directions.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _native


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def tf32_split(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """(hi, lo) TF32 parts of a contiguous fp32 CUDA tensor (numel % 4 == 0)."""
    lib = _native.load()
    hi = torch.empty_like(x)
    lo = torch.empty_like(x)
    _native.check(lib.vmscan_tf32_split(x.numel(), _ptr(x), _ptr(hi), _ptr(lo), _stream(x.device)),
                  "vmscan_tf32_split")
    return hi, lo


def tf32_split_many(xs) -> list:
    """[(hi, lo)] of several contiguous fp32 CUDA tensors (numel % 4 == 0),
    split in one launch (up to 16 per launch)."""
    lib = _native.load()
    out = [(torch.empty_like(x), torch.empty_like(x)) for x in xs]
    for a in range(0, len(xs), 16):
        chunk = list(range(a, min(a + 16, len(xs))))
        m = len(chunk)
        P = ctypes.c_void_p * m
        xp = P(*[xs[i].data_ptr() for i in chunk])
        hp = P(*[out[i][0].data_ptr() for i in chunk])
        lp = P(*[out[i][1].data_ptr() for i in chunk])
        nn = (ctypes.c_int64 * m)(*[xs[i].numel() for i in chunk])
        _native.check(lib.vmscan_tf32_split_multi(m, ctypes.cast(xp, ctypes.c_void_p), ctypes.cast(hp, ctypes.c_void_p),
                                                  ctypes.cast(lp, ctypes.c_void_p), ctypes.cast(nn, ctypes.c_void_p),
                                                  _stream(xs[0].device)), "vmscan_tf32_split_multi")
    return out


def gemm_tf32x3(a: Tuple[torch.Tensor, torch.Tensor], a_mn: bool, b: Tuple[torch.Tensor, torch.Tensor], b_mn: bool,
                m: int, n: int, k: int, out: Optional[torch.Tensor] = None, accumulate: bool = False) -> torch.Tensor:
    """C (m x n, row-major) = A B^T from split operands: A(i, j) is a[i, j]
    (a_mn False, a is m x k) or a[j, i] (a_mn True, a is k x m); B(i, j) is
    b[i, j] (b is n x k) or b[j, i] (b is k x n).  The operands may be column
    slices of wider rows (their row stride is passed); `out` (m x n, unit
    column stride, any row stride) receives C, or C is added to it when
    `accumulate`."""
    lib = _native.load()
    a_hi, a_lo = a
    b_hi, b_lo = b
    dev = a_hi.device
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=dev)
    assert out.shape == (m, n) and out.stride(1) == 1, "gemm_tf32x3: out must be (m, n) with unit column stride"
    for t in (a_hi, a_lo, b_hi, b_lo):
        assert t.stride(-1) == 1, "gemm_tf32x3: operands need unit column stride"
    ws_n = lib.vmscan_gemm_workspace_bytes(m, n, k)
    if ws_n < 0:
        _native.check(-ws_n, "vmscan_gemm_workspace_bytes")
    ws = torch.empty(int(ws_n), dtype=torch.uint8, device=dev) if ws_n > 0 else None
    _native.check(lib.vmscan_gemm_tf32x3(m, n, k, _ptr(a_hi), _ptr(a_lo), a_hi.stride(0), int(a_mn), _ptr(b_hi),
                                         _ptr(b_lo), b_hi.stride(0), int(b_mn), _ptr(out), out.stride(0),
                                         int(accumulate), _ptr(ws), int(ws_n), _stream(dev)), "vmscan_gemm_tf32x3")
    return out


def supported(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """The tensor-core path takes fp32 CUDA operands whose feature sizes are
    multiples of 4 (TMA row strides of 16 bytes)."""
    return (x.is_cuda and weight.is_cuda and x.dtype == torch.float32 and weight.dtype == torch.float32
            and x.shape[-1] % 4 == 0 and weight.shape[0] % 4 == 0 and x.numel() > 0)


class _LinearTC(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight):
        out_f, in_f = weight.shape
        x2 = x.reshape(-1, in_f).contiguous()
        t = x2.shape[0]
        xs = tf32_split(x2)
        ws = tf32_split(weight.detach().contiguous())
        y = gemm_tf32x3(xs, False, ws, False, t, out_f, in_f)
        ctx.save_for_backward(*xs, *ws)
        ctx.shape = x.shape
        return y.view(*x.shape[:-1], out_f)

    @staticmethod
    def backward(ctx, dy):
        x_hi, x_lo, w_hi, w_lo = ctx.saved_tensors
        out_f, in_f = w_hi.shape
        dy2 = dy.reshape(-1, out_f).contiguous()
        t = dy2.shape[0]
        ds = tf32_split(dy2)
        dx = dw = None
        if ctx.needs_input_grad[0]:
            # dx (t x in) = dy W: B(n = in, k = out) = W[k, n], MN-major
            dx = gemm_tf32x3(ds, False, (w_hi, w_lo), True, t, in_f, out_f).view(ctx.shape)
        if ctx.needs_input_grad[1]:
            # dW (out x in) = dy^T x: A(m = out, k = t) = dy[k, m], B(n = in, k = t) = x[k, n]
            dw = gemm_tf32x3(ds, True, (x_hi, x_lo), True, out_f, in_f, t)
        return dx, dw


def linear_tc(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """x @ weight.T on the tensor cores with fp32 accuracy (autograd-aware)."""
    return _LinearTC.apply(x, weight)
