"""The K direction branches of a (multi-directional) Mamba block as one
autograd node.

Between in_proj and out_proj each direction k runs (mamba_block.py:166-190)

    x, z   = split(xz_k)                       (in_proj output, 2 d_inner wide)
    xc     = silu(conv1d(x))                   along the direction's scan order
    x_dbc  = x_proj(xc)                        -> (dt, B, C)
    delta  = softplus(dt_proj(dt))
    y_k    = selective_scan(xc, delta, -exp(A_log), B, C, D) * silu(z)

and the block's output is out_proj(concat_k y_k) (mamba_block.py:562-566 sums
the K block outputs; one out_proj GEMM over the concatenated inner dimension
performs that sum).

Built from separate autograd nodes, PyTorch copies the branch outputs into
the concatenation, concatenates the gradients of every split (x and z of
each branch, then the K branches), and adds the scan's du to the x_proj
input gradient in a separate pass.  Here the branches write y_k straight into
their slice of one (B, L, K d_inner) output, the VJP writes dx and dz straight
into their slices of one (B, L, K 2 d_inner) gradient (the kernels take
strided outputs), the scan's dB / dC land in the slices of the x_proj-output
gradient, and the x_proj GEMM adds its input gradient onto du in place.  The
kernels and GEMMs are the same as the per-node path's; branches run on their
own CUDA streams as there.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import torch

from . import _native
from .direction import ScanDirection
from .linear import gemm_tf32x3, tf32_split, tf32_split_many
from .scan import _dir_ptr, _empty_seq, _prepare, _ptr, _strides, _tma_compatible

D_STATE = 16
PARAMS_PER_BLOCK = 7  # conv weight, conv bias, x_proj weight, dt_proj weight, dt_proj bias, A_log, D


def block_params(block) -> List[torch.Tensor]:
    return [block.conv1d.weight, block.conv1d.bias, block.x_proj.weight, block.dt_proj.weight, block.dt_proj.bias,
            block.A_log, block.D]


def _mm_tn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a^T b for tall a (K, M) and b (K, N) with small M, N (the weight
    gradients of x_proj and dt_proj, K = batch x tokens): K is split into S
    equal chunks summed after one batched GEMM, which keeps more of the GPU
    busy than cuBLAS's single skinny GEMM, and sums in a fixed order.  S is
    the largest divisor of K (at most 64) that leaves chunks of >= 256 rows:
    at K = 12544, 49 chunks of 256 (x_proj 56.6 -> 49.0 us, dt_proj 46.8 ->
    40.8 us against 16 chunks; a single GEMM took 83 / 72 us)."""
    k = a.shape[0]
    for s in range(min(64, k // 256), 1, -1):
        if k % s == 0:
            return torch.bmm(a.reshape(s, k // s, a.shape[1]).transpose(1, 2), b.reshape(s, k // s, b.shape[1])).sum(0)
    return a.t() @ b


def _tc_rows(dt_rank: int, d_inner: int) -> bool:
    """x_proj / dt_proj GEMMs run on the tensor cores when every row they read
    or write (dt_rank, dt_rank + 32, d_inner floats) is a whole number of
    16-byte units, as the GEMM's tensor maps need."""
    return dt_rank % 4 == 0 and d_inner % 4 == 0


def _stream_ptr(s: torch.cuda.Stream) -> ctypes.c_void_p:
    return ctypes.c_void_p(s.cuda_stream)


def _seq_view(t: torch.Tensor, b: int, l: int) -> torch.Tensor:
    """(B*L, C) row-major rows (possibly a column slice) as a (B, L, C) view."""
    return t.view(b, l, t.shape[-1]) if t.is_contiguous() else t.unflatten(0, (b, l))


def _run_branches_fwd(xz, meta, params, y_all, y_lo_all, need_grad, wsplits=None):
    """The K branches' forward on their streams: direction k reads its x / z
    column slices of xz and writes its scan output into its slice of y_all
    (with y_lo_all: the output's TF32 hi part into y_all and lo part into
    y_lo_all).  wsplits[k]: the TF32 parts of branch k's x_proj and dt_proj
    weights when the caller split them already.  Returns what the backward
    needs per branch."""
    lib = _native.load()
    dn, r, ksize, dirs, streams = meta["d_inner"], meta["dt_rank"], meta["d_conv"], meta["dirs"], meta["streams"]
    kb = len(dirs)
    n = D_STATE
    b, l, _ = xz.shape
    dev = xz.device
    wide = r + 2 * n
    tc = _tc_rows(r, dn)
    cur = torch.cuda.current_stream(dev)
    # A = -exp(A_log) of every branch in two multi-tensor launches
    a_all = torch._foreach_exp([params[PARAMS_PER_BLOCK * k + 5].detach() for k in range(kb)])
    torch._foreach_neg_(a_all)
    saved = []
    for k in range(kb):
        conv_w, conv_b, xproj_w, dt_w, dt_b, _, d_skip = params[PARAMS_PER_BLOCK * k:PARAMS_PER_BLOCK * (k + 1)]
        s = streams[k]
        s.wait_stream(cur)
        with torch.cuda.stream(s):
            sp = _stream_ptr(s)
            dptr = _dir_ptr(dirs[k])
            x = xz[:, :, 2 * dn * k:2 * dn * k + dn]
            z = xz[:, :, 2 * dn * k + dn:2 * dn * (k + 1)]
            if not (_tma_compatible(x) and _tma_compatible(z)):
                x, z = _prepare(x), _prepare(z)
            cw = conv_w.detach().contiguous()
            cb = conv_b.detach().contiguous()
            xc = _empty_seq(b, l, dn, dev)
            # with the tensor-core x_proj the conv also writes xc's TF32 parts (its GEMM operand)
            xc_s = (_empty_seq(b, l, dn, dev), _empty_seq(b, l, dn, dev)) if tc else (None, None)
            _native.check(lib.vmscan_conv1d_silu_fwd(b, l, dn, ksize, _ptr(x), _strides(x), _ptr(cw), _ptr(cb),
                                                     _ptr(xc), _strides(xc), _ptr(xc_s[0]), _ptr(xc_s[1]), dptr,
                                                     sp), "vmscan_conv1d_silu_fwd")
            if tc:
                xc_s = (xc_s[0].view(b * l, dn), xc_s[1].view(b * l, dn))
                wx_s = wsplits[k][0] if wsplits is not None else tf32_split(xproj_w.detach().contiguous())
                xdbc = gemm_tf32x3(xc_s, False, wx_s, False, b * l, wide, dn)
            else:
                xdbc = torch.mm(xc.reshape(b * l, dn), xproj_w.detach().t())  # (B L, r + 2n)
            dw_ = dt_w.detach().contiguous()
            db_ = dt_b.detach().contiguous()
            delta = _empty_seq(b, l, dn, dev)
            _native.check(lib.vmscan_dt_softplus_fwd(b * l, r, dn, _ptr(xdbc), wide, _ptr(dw_), _ptr(db_),
                                                     _ptr(delta), delta.stride(1), sp), "vmscan_dt_softplus_fwd")
            a = a_all[k]
            bmat = _prepare(_seq_view(xdbc[:, r:r + n], b, l))
            cmat = _prepare(_seq_view(xdbc[:, r + n:], b, l))
            dsk = d_skip.detach().contiguous()
            y = y_all[:, :, dn * k:dn * (k + 1)]
            y_lo = y_lo_all[:, :, dn * k:dn * (k + 1)] if y_lo_all is not None else None
            ckpt = None
            if need_grad:
                n_ck = lib.vmscan_ckpt_elems(b, l, dn, D_STATE, dptr)
                if n_ck < 0:
                    _native.check(-n_ck, "vmscan_ckpt_elems")
                ckpt = torch.empty(n_ck, dtype=torch.float32, device=dev)
            fws_n = lib.vmscan_fwd_workspace_bytes(b, l, dn, D_STATE, dptr)
            if fws_n < 0:
                _native.check(-fws_n, "vmscan_fwd_workspace_bytes")
            fws = torch.empty(int(fws_n), dtype=torch.uint8, device=dev) if fws_n > 0 else None
            _native.check(lib.vmscan_fwd(b, l, dn, D_STATE, _ptr(xc), _strides(xc), _ptr(delta), _strides(delta),
                                         _ptr(a), _ptr(bmat), _strides(bmat), _ptr(cmat), _strides(cmat),
                                         _ptr(dsk), _ptr(z), _strides(z), _ptr(y), _strides(y), _ptr(y_lo),
                                         _ptr(ckpt), dptr, _ptr(fws), int(fws_n), sp), "vmscan_fwd")
            saved.append((x, z, cw, cb, xc, xdbc, dw_, db_, delta, a, bmat, cmat, dsk, ckpt, xc_s,
                          wsplits[k] if wsplits is not None else None))
    for s in streams[:kb]:
        cur.wait_stream(s)
    return saved


def _run_branches_bwd(saved, xproj, meta, dy_all, dxz, dxz_lo):
    """The K branches' VJP on their streams: direction k reads its slice of
    dy_all and writes dx / dz into its slices of dxz (with dxz_lo: their TF32
    hi parts into dxz and lo parts into dxz_lo).  Returns the parameter
    gradients in block_params order, branch after branch."""
    lib = _native.load()
    dn, r, ksize, dirs, streams = meta["d_inner"], meta["dt_rank"], meta["d_conv"], meta["dirs"], meta["streams"]
    kb = len(dirs)
    n = D_STATE
    b, l, _ = dy_all.shape
    dev = dy_all.device
    wide = r + 2 * n
    tc = _tc_rows(r, dn)
    cur = torch.cuda.current_stream(dev)
    grads: List[Optional[torch.Tensor]] = [None] * (PARAMS_PER_BLOCK * kb)
    for k in range(kb):
        x, z, cw, cb, xc, xdbc, dw_, db_, delta, a, bmat, cmat, dsk, ckpt, xc_s, wsp = saved[k]
        xproj_w = xproj[k].detach()
        s = streams[k]
        s.wait_stream(cur)
        with torch.cuda.stream(s):
            sp = _stream_ptr(s)
            dptr = _dir_ptr(dirs[k])
            dy = _prepare(dy_all[:, :, dn * k:dn * (k + 1)])
            du = _empty_seq(b, l, dn, dev)
            ddelta = _empty_seq(b, l, dn, dev)
            dA = torch.empty((dn, n), dtype=torch.float32, device=dev)
            dD = torch.empty((dn,), dtype=torch.float32, device=dev)
            dxdbc = torch.empty((b * l, wide), dtype=torch.float32, device=dev)
            dB = _seq_view(dxdbc[:, r:r + n], b, l)
            dC = _seq_view(dxdbc[:, r + n:], b, l)
            dz = dxz[:, :, 2 * dn * k + dn:2 * dn * (k + 1)]
            dz_lo = dxz_lo[:, :, 2 * dn * k + dn:2 * dn * (k + 1)] if dxz_lo is not None else None
            ws_n = lib.vmscan_bwd_workspace_bytes(b, l, dn, D_STATE, dptr, 0)
            if ws_n < 0:
                _native.check(-ws_n, "vmscan_bwd_workspace_bytes")
            ws = torch.empty(max(int(ws_n), 256), dtype=torch.uint8, device=dev)
            _native.check(lib.vmscan_bwd(b, l, dn, D_STATE, _ptr(xc), _strides(xc), _ptr(delta), _strides(delta),
                                         _ptr(a), _ptr(bmat), _strides(bmat), _ptr(cmat), _strides(cmat),
                                         _ptr(dsk), _ptr(z), _strides(z), _ptr(ckpt), _ptr(dy), _strides(dy),
                                         _ptr(du), _strides(du), _ptr(ddelta), _strides(ddelta), _ptr(dA),
                                         _ptr(dB), _strides(dB), _ptr(dC), _strides(dC), _ptr(dD), _ptr(dz),
                                         _strides(dz), _ptr(dz_lo), dptr, _ptr(ws), ws.numel(), sp),
                          "vmscan_bwd")
            # dt_proj + softplus: dpre (for the tensor cores: its TF32 parts), then its
            # GEMMs; dbias from the kernel's partial sums
            t = b * l
            dpre = _empty_seq(b, l, dn, dev)
            dpre_lo = _empty_seq(b, l, dn, dev) if tc else None
            part = torch.empty((lib.vmscan_dt_softplus_bias_rows(t), dn), dtype=torch.float32, device=dev)
            _native.check(lib.vmscan_dt_softplus_bwd(t, r, dn, _ptr(xdbc), wide, _ptr(dw_), _ptr(db_),
                                                     _ptr(ddelta), ddelta.stride(1), _ptr(dpre), dpre.stride(1),
                                                     _ptr(dpre_lo), _ptr(part), sp), "vmscan_dt_softplus_bwd")
            g_dt_b = torch.empty((dn,), dtype=torch.float32, device=dev)
            _native.check(lib.vmscan_sum_rows(part.shape[0], dn, _ptr(part), _ptr(g_dt_b), sp), "vmscan_sum_rows")
            du2 = du.view(t, dn)
            if tc:
                dpre_s = (dpre.view(t, dn), dpre_lo.view(t, dn))
                xdbc_s = tf32_split(xdbc)
                # dt_proj input gradient straight into its slice of dx_dbc: dpre W_dt
                wdt_s = wsp[1] if wsp is not None else tf32_split(dw_)
                gemm_tf32x3(dpre_s, False, wdt_s, True, t, r, dn, out=dxdbc[:, :r])
                # dt_proj weight gradient dpre^T x_dbc[:, :r] (both read MN-major)
                g_dt_w = gemm_tf32x3(dpre_s, True, (xdbc_s[0][:, :r], xdbc_s[1][:, :r]), True, dn, r, t)
                # x_proj: its input gradient lands on du in place (du += dx_dbc W_x)
                dxdbc_s = tf32_split(dxdbc)
                wx_s = wsp[0] if wsp is not None else tf32_split(xproj_w.contiguous())
                gemm_tf32x3(dxdbc_s, False, wx_s, True, t, dn, wide, out=du2, accumulate=True)
                g_xproj = gemm_tf32x3(dxdbc_s, True, xc_s, True, wide, dn, t)
            else:
                dpre2 = dpre.reshape(t, dn)
                dxdbc[:, :r].copy_(torch.mm(dpre2, dw_))
                g_dt_w = _mm_tn(dpre2, xdbc[:, :r])
                # x_proj: its input gradient lands on du in place (du += dx_dbc W)
                du2.addmm_(dxdbc, xproj_w)
                g_xproj = _mm_tn(dxdbc, xc.reshape(t, dn))
            # conv1d + SiLU: dx straight into its slice of dxz
            dx = dxz[:, :, 2 * dn * k:2 * dn * k + dn]
            dx_lo = dxz_lo[:, :, 2 * dn * k:2 * dn * k + dn] if dxz_lo is not None else None
            g_cw = torch.empty_like(cw)
            g_cb = torch.empty_like(cb)
            cws_n = lib.vmscan_conv1d_bwd_workspace_bytes(b, l, dn, ksize)
            if cws_n < 0:
                _native.check(-cws_n, "vmscan_conv1d_bwd_workspace_bytes")
            cws = torch.empty(int(cws_n), dtype=torch.uint8, device=dev)
            _native.check(lib.vmscan_conv1d_silu_bwd(b, l, dn, ksize, _ptr(x), _strides(x), _ptr(cw), _ptr(cb),
                                                     _ptr(du), _strides(du), _ptr(dx), _strides(dx), _ptr(dx_lo),
                                                     _ptr(g_cw), _ptr(g_cb), dptr, _ptr(cws), cws.numel(), sp),
                          "vmscan_conv1d_silu_bwd")
            grads[PARAMS_PER_BLOCK * k:PARAMS_PER_BLOCK * (k + 1)] = [g_cw, g_cb, g_xproj, g_dt_w, g_dt_b, dA,
                                                                      dD]
    for s in streams[:kb]:
        cur.wait_stream(s)
    # A = -exp(A_log): dA_log = dA * A, every branch in one multi-tensor launch
    g_alogs = torch._foreach_mul([grads[PARAMS_PER_BLOCK * k + 5] for k in range(kb)], [sv[9] for sv in saved])
    for k in range(kb):
        grads[PARAMS_PER_BLOCK * k + 5] = g_alogs[k]
    return grads


class _BranchesFn(torch.autograd.Function):
    """xz (in_proj output, B x L x K 2 d_inner) -> y_all (B x L x K d_inner)."""

    @staticmethod
    def forward(ctx, xz, meta, *params):
        b, l, _ = xz.shape
        kb = len(meta["dirs"])
        y_all = _empty_seq(b, l, kb * meta["d_inner"], xz.device)
        need_grad = any(ctx.needs_input_grad)
        saved = _run_branches_fwd(xz, meta, params, y_all, None, need_grad)
        if need_grad:
            ctx.saved = saved
            ctx.xproj = [params[PARAMS_PER_BLOCK * k + 2] for k in range(kb)]
            ctx.meta = meta
        return y_all

    @staticmethod
    def backward(ctx, dy_all):
        meta = ctx.meta
        b, l, _ = dy_all.shape
        dxz = _empty_seq(b, l, len(meta["dirs"]) * 2 * meta["d_inner"], dy_all.device)
        grads = _run_branches_bwd(ctx.saved, ctx.xproj, meta, dy_all, dxz, None)
        ctx.saved = None
        return (dxz, None, *grads)


class _BlockCoreFn(torch.autograd.Function):
    """h (B x L x E) -> out_proj(concat_k branch_k(in_proj(h))) as one node.

    in_proj and out_proj run on the tensor-core GEMM with the block's
    concatenated weights (w_in: K 2 d_inner x E, w_out: E x K d_inner), and
    the tensors between them never exist as fp32 where only a GEMM reads
    them: the scans write y_all as its TF32 parts (the out_proj operand, kept
    for out_proj's weight gradient), and the scan and conv VJPs write dxz, the
    in_proj output gradient, as its TF32 parts (the operand of in_proj's input
    and weight gradients).  Only h, the block output's gradient and the
    weights go through separate split passes."""

    @staticmethod
    def forward(ctx, h, w_in, w_out, meta, *params):
        b, l, e = h.shape
        kb, dn = len(meta["dirs"]), meta["d_inner"]
        t = b * l
        h_s = tf32_split(h.reshape(t, e).contiguous())
        # every weight of the block split in one launch: in_proj, out_proj, then
        # each branch's x_proj and dt_proj
        ws = [w_in.detach().contiguous(), w_out.detach().contiguous()]
        if _tc_rows(meta["dt_rank"], dn):
            for k in range(kb):
                ws += [params[PARAMS_PER_BLOCK * k + 2].detach().contiguous(),
                       params[PARAMS_PER_BLOCK * k + 3].detach().contiguous()]
        splits = tf32_split_many(ws)
        win_s, wout_s = splits[0], splits[1]
        wsplits = [(splits[2 + 2 * k], splits[3 + 2 * k]) for k in range(kb)] if len(splits) > 2 else None
        xz = gemm_tf32x3(h_s, False, win_s, False, t, kb * 2 * dn, e).view(b, l, kb * 2 * dn)
        y_hi = _empty_seq(b, l, kb * dn, h.device)
        y_lo = _empty_seq(b, l, kb * dn, h.device)
        need_grad = any(ctx.needs_input_grad)
        saved = _run_branches_fwd(xz, meta, params, y_hi, y_lo, need_grad, wsplits)
        y_s = (y_hi.view(t, kb * dn), y_lo.view(t, kb * dn))
        out = gemm_tf32x3(y_s, False, wout_s, False, t, e, kb * dn).view(b, l, e)
        if need_grad:
            ctx.saved = saved
            ctx.xproj = [params[PARAMS_PER_BLOCK * k + 2] for k in range(kb)]
            ctx.meta = meta
            ctx.parts = (h_s, win_s, y_s, wout_s)
        return out

    @staticmethod
    def backward(ctx, dout):
        meta = ctx.meta
        h_s, win_s, y_s, wout_s = ctx.parts
        b, l, e = dout.shape
        kb, dn = len(meta["dirs"]), meta["d_inner"]
        t = b * l
        dev = dout.device
        d_s = tf32_split(dout.reshape(t, e).contiguous())
        # out_proj: weight gradient dout^T y, input gradient dout W_out (W_out read MN-major)
        g_wout = gemm_tf32x3(d_s, True, y_s, True, e, kb * dn, t)
        dy_all = gemm_tf32x3(d_s, False, wout_s, True, t, kb * dn, e).view(b, l, kb * dn)
        dxz_hi = _empty_seq(b, l, kb * 2 * dn, dev)
        dxz_lo = _empty_seq(b, l, kb * 2 * dn, dev)
        grads = _run_branches_bwd(ctx.saved, ctx.xproj, meta, dy_all, dxz_hi, dxz_lo)
        dxz_s = (dxz_hi.view(t, kb * 2 * dn), dxz_lo.view(t, kb * 2 * dn))
        # in_proj: input gradient dxz W_in (W_in read MN-major), weight gradient dxz^T h
        dh = gemm_tf32x3(dxz_s, False, win_s, True, t, e, kb * 2 * dn).view(b, l, e)
        g_win = gemm_tf32x3(dxz_s, True, h_s, True, kb * 2 * dn, e, t)
        ctx.saved = ctx.parts = None
        return (dh, g_win, g_wout, None, *grads)


def block_core_ok(blocks: Sequence, h: torch.Tensor) -> bool:
    """_BlockCoreFn applies when every row its GEMMs read or write (E, K 2
    d_inner, K d_inner floats) is a whole number of 16-byte units."""
    b0 = blocks[0]
    return (h.is_cuda and h.dtype == torch.float32 and h.shape[-1] % 4 == 0 and b0.d_inner % 4 == 0
            and _tc_rows(b0.dt_rank, b0.d_inner) and h.numel() > 0)


def block_core_forward(blocks: Sequence, directions: Sequence[Optional[ScanDirection]], h: torch.Tensor,
                       w_in: torch.Tensor, w_out: torch.Tensor, streams: Sequence[torch.cuda.Stream]) -> torch.Tensor:
    """sum_k block_k(h, direction_k) for K MambaBlocks as one autograd node
    (_BlockCoreFn); w_in / w_out are the blocks' in_proj / out_proj weights
    concatenated (torch.cat, so their gradients reach every block)."""
    b0 = blocks[0]
    meta = {"d_inner": b0.d_inner, "dt_rank": b0.dt_rank, "d_conv": b0.d_conv, "dirs": list(directions),
            "streams": list(streams)}
    params = [p for blk in blocks for p in block_params(blk)]
    return _BlockCoreFn.apply(h, w_in, w_out, meta, *params)


def branches_forward(blocks: Sequence, directions: Sequence[Optional[ScanDirection]], xz: torch.Tensor,
                     streams: Sequence[torch.cuda.Stream]) -> torch.Tensor:
    """y = concat_k scan_branch_k(xz_k) for K MambaBlocks sharing one in_proj
    output xz (B, L, K 2 d_inner), as one autograd node; returns (B, L, K d_inner)."""
    b0 = blocks[0]
    meta = {"d_inner": b0.d_inner, "dt_rank": b0.dt_rank, "d_conv": b0.d_conv, "dirs": list(directions),
            "streams": list(streams)}
    params = [p for blk in blocks for p in block_params(blk)]
    return _BranchesFn.apply(xz.contiguous(), meta, *params)
