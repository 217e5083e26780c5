"""Selective scan and direction-aware conv1d+SiLU as autograd functions over libvmscan.so.

`selective_scan_cuda(x, delta, A, B, C, D, z=None, direction=None)` is the
drop-in for the reference's scan functions, which share the positional
signature `scan(x, delta, A, B, C, D) -> y` (mlx_vision_mamba/mamba_block.py:20-74,
mamba_metal_fused.py:253-267).  Two keyword extensions: `z` fuses the gate
`y * silu(z)` of MambaBlock (mamba_block.py:190) into the kernel, and
`direction` folds a multi-directional scan order into the kernel's indexing.

The custom VJP mirrors `_fused_scan_core.vjp` (mamba_metal_fused.py:236-250):
it returns gradients for all primals (and dz), reducing dA, dB, dC and dD on
the device.  Instead of recomputing the full forward and storing h for every
step (a (B, L, D, N) buffer in the reference), the forward saves the state at
the end of every 16-step box and the VJP recomputes each box from it.

There is no CPU path: inputs must be CUDA tensors and libvmscan.so must load.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _native
from .direction import ScanDirection

D_STATE = 16


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _strides(t: Optional[torch.Tensor]) -> _native.Strides:
    if t is None:
        return _native.Strides(0, 0)
    return _native.Strides(t.stride(0), t.stride(1))


# Sequence tensors travel as fp32 (the reference's precision) or bf16 (the
# bf16 I/O entry points); TMA strides are whole 16-byte multiples, i.e. 4 fp32
# or 8 bf16 elements.
_SEQ_DTYPES = (torch.float32, torch.bfloat16)


def _align_elems(dtype: torch.dtype) -> int:
    return 16 // (4 if dtype == torch.float32 else 2)


def _tma_compatible(t: torch.Tensor, dtype: torch.dtype = torch.float32) -> bool:
    """True when the (B, L, C) view meets the TMA rules of include/vmscan.h."""
    if t.dtype != dtype or t.dim() != 3 or t.stride(2) != 1 and t.size(2) > 1:
        return False
    if t.data_ptr() % 16:
        return False
    q = _align_elems(dtype)
    b, l, _ = t.shape
    if l > 1 and (t.stride(1) <= 0 or t.stride(1) % q):
        return False
    if b > 1 and (t.stride(0) <= 0 or t.stride(0) % q):
        return False
    return True


def _empty_seq(b: int, l: int, c: int, device, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Uninitialised (b, l, c) view whose storage rows are padded to a whole
    16 bytes, as the TMA rules of include/vmscan.h require."""
    q = _align_elems(dtype)
    cp = (c + q - 1) // q * q
    buf = torch.empty((b, l, cp), dtype=dtype, device=device)
    return buf if cp == c else buf[:, :, :c]


def _prepare(t: torch.Tensor, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Return a TMA-compatible view of t in `dtype`, copying only when needed.

    Strided views such as the reference's `xz[:, :, :d_inner]` slices pass
    through untouched; a copy is made only for another dtype, a non-unit
    channel stride, or strides that are not whole 16-byte multiples (then the
    channel dim is padded in storage).
    """
    if t.dtype != dtype:
        t = t.to(dtype)
    if _tma_compatible(t, dtype):
        return t
    b, l, c = t.shape
    out = _empty_seq(b, l, c, t.device, dtype)
    out.copy_(t)
    return out


def _dir_ptr(direction: Optional[ScanDirection]):
    if direction is None:
        return None
    return ctypes.byref(direction.to_native())


def _check_inputs(x, delta, A, B, C, D, z):
    for name, t in (("x", x), ("delta", delta), ("A", A), ("B", B), ("C", C), ("D", D)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError(f"selective_scan_cuda: `{name}` must be a CUDA tensor (there is no CPU path)")
    if z is not None and not z.is_cuda:
        raise RuntimeError("selective_scan_cuda: `z` must be a CUDA tensor")
    if x.dim() != 3:
        raise ValueError(f"x must be (B, L, D_inner), got {tuple(x.shape)}")
    bt, l, dn = x.shape
    if A.dim() != 2 or A.shape[0] != dn:
        raise ValueError(f"A must be (D_inner, N), got {tuple(A.shape)}")
    n = A.shape[1]
    if n != D_STATE:
        raise ValueError(f"d_state must be {D_STATE} (the kernel holds a 16-float state), got {n}")
    if tuple(delta.shape) != (bt, l, dn):
        raise ValueError(f"delta must be {(bt, l, dn)}, got {tuple(delta.shape)}")
    for name, t in (("B", B), ("C", C)):
        if tuple(t.shape) != (bt, l, n):
            raise ValueError(f"{name} must be {(bt, l, n)}, got {tuple(t.shape)}")
    if tuple(D.shape) != (dn,):
        raise ValueError(f"D must be ({dn},), got {tuple(D.shape)}")
    if z is not None and tuple(z.shape) != (bt, l, dn):
        raise ValueError(f"z must be {(bt, l, dn)}, got {tuple(z.shape)}")


class _SelectiveScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, delta, A, B, C, D, z, direction):
        bt, l, dn = x.shape
        sd = torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float32
        ctx.has_z = z is not None
        ctx.param_dtypes = (A.dtype, D.dtype)
        ctx.empty = bt * l * dn == 0
        if ctx.empty:
            # nothing to scan: zero-size y (or, for D_inner > 0 with no tokens,
            # no rows); every gradient is zero, dA / dD included
            ctx.shapes = (x.shape, A.shape, B.shape, D.shape)
            ctx.sd = sd
            return torch.zeros((bt, l, dn), dtype=sd, device=x.device)
        lib = _native.load()
        u_ = _prepare(x, sd)
        dt_ = _prepare(delta, sd)
        B_ = _prepare(B, sd)
        C_ = _prepare(C, sd)
        z_ = _prepare(z, sd) if z is not None else None
        A_ = A.detach().float().contiguous()
        D_ = D.detach().float().contiguous()
        y = _empty_seq(bt, l, dn, x.device, sd)
        need_grad = any(ctx.needs_input_grad[:7])
        dptr = _dir_ptr(direction)
        ckpt = None
        if need_grad:
            n_ck = lib.vmscan_ckpt_elems(bt, l, dn, D_STATE, dptr)
            if n_ck < 0:
                _native.check(-n_ck, "vmscan_ckpt_elems")
            ckpt = torch.empty(n_ck, dtype=torch.float32, device=x.device)
        fws_n = lib.vmscan_fwd_workspace_bytes(bt, l, dn, D_STATE, dptr)
        if fws_n < 0:
            _native.check(-fws_n, "vmscan_fwd_workspace_bytes")
        fws = torch.empty(int(fws_n), dtype=torch.uint8, device=x.device) if fws_n > 0 else None
        head = (bt, l, dn, D_STATE, _ptr(u_), _strides(u_), _ptr(dt_), _strides(dt_), _ptr(A_), _ptr(B_),
                _strides(B_), _ptr(C_), _strides(C_), _ptr(D_), _ptr(z_), _strides(z_), _ptr(y), _strides(y))
        tail = (_ptr(ckpt), dptr, _ptr(fws), int(fws_n), _stream(x))
        if sd == torch.bfloat16:
            st = lib.vmscan_fwd_bf16(*head, *tail)
        else:
            st = lib.vmscan_fwd(*head, None, *tail)  # y_lo: the fp32 output itself
        _native.check(st, "vmscan_fwd_bf16" if sd == torch.bfloat16 else "vmscan_fwd")
        if need_grad:
            ctx.save_for_backward(u_, dt_, A_, B_, C_, D_, z_, ckpt)
        ctx.direction = direction
        return y

    @staticmethod
    def backward(ctx, dy):
        if ctx.empty:
            xs, As, Bs, Ds = ctx.shapes
            dev = dy.device
            seq = torch.zeros(xs, dtype=ctx.sd, device=dev)
            a_dt, d_dt = ctx.param_dtypes
            return (seq, seq.clone(), torch.zeros(As, dtype=a_dt, device=dev),
                    torch.zeros(Bs, dtype=ctx.sd, device=dev), torch.zeros(Bs, dtype=ctx.sd, device=dev),
                    torch.zeros(Ds, dtype=d_dt, device=dev), seq.clone() if ctx.has_z else None, None)
        lib = _native.load()
        u_, dt_, A_, B_, C_, D_, z_, ckpt = ctx.saved_tensors
        bt, l, dn = u_.shape
        dev = u_.device
        sd = u_.dtype
        dy_ = _prepare(dy, sd)
        f32 = dict(dtype=torch.float32, device=dev)
        du = _empty_seq(bt, l, dn, dev, sd)
        ddelta = _empty_seq(bt, l, dn, dev, sd)
        dA = torch.empty((dn, D_STATE), **f32)
        dB = torch.empty((bt, l, D_STATE), dtype=sd, device=dev)
        dC = torch.empty((bt, l, D_STATE), dtype=sd, device=dev)
        dD = torch.empty((dn,), **f32)
        dz = _empty_seq(bt, l, dn, dev, sd) if ctx.has_z else None
        dptr = _dir_ptr(ctx.direction)
        ws_bytes = lib.vmscan_bwd_workspace_bytes(bt, l, dn, D_STATE, dptr, 0)
        if ws_bytes < 0:
            _native.check(-ws_bytes, "vmscan_bwd_workspace_bytes")
        ws = torch.empty(max(int(ws_bytes), 256), dtype=torch.uint8, device=dev)
        head = (bt, l, dn, D_STATE, _ptr(u_), _strides(u_), _ptr(dt_), _strides(dt_), _ptr(A_), _ptr(B_),
                _strides(B_), _ptr(C_), _strides(C_), _ptr(D_), _ptr(z_), _strides(z_), _ptr(ckpt), _ptr(dy_),
                _strides(dy_), _ptr(du), _strides(du), _ptr(ddelta), _strides(ddelta), _ptr(dA), _ptr(dB),
                _strides(dB), _ptr(dC), _strides(dC), _ptr(dD), _ptr(dz), _strides(dz))
        tail = (dptr, _ptr(ws), ws.numel(), _stream(u_))
        if sd == torch.bfloat16:
            st = lib.vmscan_bwd_bf16(*head, *tail)
        else:
            st = lib.vmscan_bwd(*head, None, *tail)  # dz_lo: dz itself
        _native.check(st, "vmscan_bwd_bf16" if sd == torch.bfloat16 else "vmscan_bwd")
        a_dt, d_dt = ctx.param_dtypes
        return du, ddelta, dA.to(a_dt), dB, dC, dD.to(d_dt), dz, None


def selective_scan_cuda(
    x: torch.Tensor,
    delta: torch.Tensor,
    A: torch.Tensor,
    B: torch.Tensor,
    C: torch.Tensor,
    D: torch.Tensor,
    z: Optional[torch.Tensor] = None,
    direction: Optional[ScanDirection] = None,
) -> torch.Tensor:
    """Fused selective scan (S6) on sm_100a.

    Args (shapes as in mlx_vision_mamba/mamba_block.py:35-40):
        x:     (B, L, D_inner)   input after conv1d + SiLU
        delta: (B, L, D_inner)   discretisation steps
        A:     (D_inner, 16)     state matrix (negative)
        B, C:  (B, L, 16)        input / output projections
        D:     (D_inner,)        skip
        z:     optional (B, L, D_inner) gate; returns y * silu(z)
        direction: optional ScanDirection; tokens are visited in that order
            and y is returned in token order.
    Returns y (B, L, D_inner): fp32, or bf16 when x is bf16.  With a bf16 x
    the sequence tensors (x, delta, B, C, z) are read as bf16 (cast if they
    are not) and y and their gradients are bf16; A, D, the recurrent state and
    all arithmetic stay fp32.  Any other dtype is computed in fp32.
    A zero batch, sequence length or channel count launches nothing: y is
    zero-size and every gradient is zero.
    """
    _check_inputs(x, delta, A, B, C, D, z)
    if direction is not None and direction.grid:
        n = 1
        for g in direction.grid:
            n *= g
        if n != x.shape[1]:
            raise ValueError(f"direction grid {direction.grid} does not cover {x.shape[1]} tokens")
    return _SelectiveScanFn.apply(x, delta, A, B, C, D, z, direction)


# Reference entry-point names (mlx_vision_mamba/__init__.py:14-19) bound to the
# CUDA implementation, so code importing them keeps working.
def selective_scan(x, delta, A, B, C, D):
    return selective_scan_cuda(x, delta, A, B, C, D)


selective_scan_metal = selective_scan
selective_scan_metal_trainable = selective_scan
selective_scan_metal_fused = selective_scan


class _ConvSiluFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, direction):
        lib = _native.load()
        bt, l, c = x.shape
        k = weight.shape[1]
        x_ = _prepare(x)
        w_ = weight.detach().float().contiguous()
        b_ = bias.detach().float().contiguous()
        out = _empty_seq(bt, l, c, x.device)
        st = lib.vmscan_conv1d_silu_fwd(
            bt, l, c, k, _ptr(x_), _strides(x_), _ptr(w_), _ptr(b_), _ptr(out), _strides(out), None, None,
            _dir_ptr(direction), _stream(x),
        )
        _native.check(st, "vmscan_conv1d_silu_fwd")
        ctx.save_for_backward(x_, w_, b_)
        ctx.direction = direction
        return out

    @staticmethod
    def backward(ctx, dout):
        lib = _native.load()
        x_, w_, b_ = ctx.saved_tensors
        bt, l, c = x_.shape
        k = w_.shape[1]
        dout_ = _prepare(dout)
        dx = _empty_seq(bt, l, c, x_.device)
        dw = torch.empty_like(w_)
        db = torch.empty_like(b_)
        ws_bytes = lib.vmscan_conv1d_bwd_workspace_bytes(bt, l, c, k)
        if ws_bytes < 0:
            _native.check(-ws_bytes, "vmscan_conv1d_bwd_workspace_bytes")
        ws = torch.empty(int(ws_bytes), dtype=torch.uint8, device=x_.device)
        st = lib.vmscan_conv1d_silu_bwd(
            bt, l, c, k, _ptr(x_), _strides(x_), _ptr(w_), _ptr(b_), _ptr(dout_), _strides(dout_),
            _ptr(dx), _strides(dx), None, _ptr(dw), _ptr(db), _dir_ptr(ctx.direction), _ptr(ws), ws.numel(),
            _stream(x_),
        )
        _native.check(st, "vmscan_conv1d_silu_bwd")
        return dx, dw, db, None


def conv1d_silu_cuda(
    x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, direction: Optional[ScanDirection] = None
) -> torch.Tensor:
    """silu(causal depthwise conv1d(x)) along the scan order of `direction`.

    x: (B, L, C) CUDA fp32, channel-last as in MLX; weight: (C, K, 1) in MLX's
    Conv1d layout; bias: (C,).  Equivalent to `silu(conv1d(x_perm)[:, :L])`
    un-permuted (mlx_vision_mamba/mamba_block.py:129-132,170-171).
    """
    if not (x.is_cuda and weight.is_cuda and bias.is_cuda):
        raise RuntimeError("conv1d_silu_cuda: inputs must be CUDA tensors (there is no CPU path)")
    if x.dim() != 3 or weight.dim() != 3 or weight.shape[0] != x.shape[2] or weight.shape[2] != 1:
        raise ValueError(f"bad shapes x={tuple(x.shape)} weight={tuple(weight.shape)}")
    return _ConvSiluFn.apply(x, weight, bias, direction)


def _token_rows(t: torch.Tensor) -> torch.Tensor:
    """t (B, L, C) as ntok = B*L rows of C floats with one row stride (a view
    when the layout allows it, else a contiguous copy)."""
    if t.dtype != torch.float32:
        t = t.float()
    b, l, c = t.shape
    if t.stride(2) == 1 and t.stride(1) >= c and (b == 1 or t.stride(0) == l * t.stride(1)):
        return t
    return t.contiguous()


class _DtSoftplusFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias):
        lib = _native.load()
        b, l, r = x.shape
        dn = weight.shape[0]
        x_ = _token_rows(x)
        w_ = weight.detach().float().contiguous()
        b_ = bias.detach().float().contiguous()
        delta = _empty_seq(b, l, dn, x.device)
        st = lib.vmscan_dt_softplus_fwd(b * l, r, dn, _ptr(x_), x_.stride(1), _ptr(w_), _ptr(b_), _ptr(delta),
                                        delta.stride(1), _stream(x))
        _native.check(st, "vmscan_dt_softplus_fwd")
        ctx.save_for_backward(x_, w_, b_)
        return delta

    @staticmethod
    def backward(ctx, ddelta):
        lib = _native.load()
        x_, w_, b_ = ctx.saved_tensors
        b, l, r = x_.shape
        dn = w_.shape[0]
        g_in = _token_rows(ddelta)
        dpre = _empty_seq(b, l, dn, x_.device)
        # dbias: the kernel sums dpre over each group of tokens it handles;
        # vmscan_sum_rows adds the rows of those partials in a fixed order
        part = torch.empty((lib.vmscan_dt_softplus_bias_rows(b * l), dn), dtype=torch.float32, device=x_.device)
        st = lib.vmscan_dt_softplus_bwd(b * l, r, dn, _ptr(x_), x_.stride(1), _ptr(w_), _ptr(b_), _ptr(g_in),
                                        g_in.stride(1), _ptr(dpre), dpre.stride(1), None, _ptr(part), _stream(x_))
        _native.check(st, "vmscan_dt_softplus_bwd")
        g2 = dpre.reshape(b * l, dn)
        dx = (g2 @ w_).reshape(b, l, r)
        dw = g2.t() @ x_.reshape(b * l, r)
        db = torch.empty((dn,), dtype=torch.float32, device=x_.device)
        _native.check(lib.vmscan_sum_rows(part.shape[0], dn, _ptr(part), _ptr(db), _stream(x_)), "vmscan_sum_rows")
        return dx, dw, db


def dt_softplus_cuda(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """delta = log(1 + exp(x @ weight.T + bias)) in one kernel (the reference's
    `dt_proj` followed by its softplus, mlx_vision_mamba/mamba_block.py:180-181).

    x: (B, L, dt_rank) CUDA fp32 (the dt columns of x_dbc, a strided view is
    fine); weight: (d_inner, dt_rank) and bias: (d_inner,) of nn.Linear.
    Returns (B, L, d_inner).  The backward forms dpre = ddelta * sigmoid(pre)
    in a kernel and leaves dx, dweight, dbias to cuBLAS GEMMs / a reduction.
    """
    if not (x.is_cuda and weight.is_cuda and bias.is_cuda):
        raise RuntimeError("dt_softplus_cuda: inputs must be CUDA tensors (there is no CPU path)")
    if x.dim() != 3 or weight.dim() != 2 or weight.shape[1] != x.shape[2] or bias.shape != (weight.shape[0],):
        raise ValueError(f"bad shapes x={tuple(x.shape)} weight={tuple(weight.shape)} bias={tuple(bias.shape)}")
    return _DtSoftplusFn.apply(x, weight, bias)


def device_status(device: Optional[torch.device] = None, clear: bool = True) -> int:
    """Synchronise the current stream and return the sticky device status (0 = ok)."""
    lib = _native.load()
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    return int(lib.vmscan_device_status(ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream), int(clear)))
