"""Selective-scan oracle: the reference's sequential and chunked scans on the CPU.

TEST INFRASTRUCTURE ONLY (the parity checker and the CPU baseline).

Both functions keep the reference's order of operations: discretise the whole
sequence into two (B, L, D, N) tensors, then walk the recurrence one step at a
time, stack, and add the skip term last.  Any float dtype works; fp32 is the
reference's arithmetic, fp64 is used to measure how far fp32 results are from
the exact answer.
"""

from __future__ import annotations

import torch


def _discretize(x, delta, A, B):
    """deltaA = exp(delta * A), deltaB_x = delta * B * x  (mamba_block.py:48-59)."""
    d = delta.unsqueeze(-1)                      # (B, L, D, 1)
    deltaA = torch.exp(d * A[None, None])        # (B, L, D, N)
    deltaB_x = d * B.unsqueeze(2) * x.unsqueeze(-1)
    return deltaA, deltaB_x


def selective_scan(x, delta, A, B, C, D):
    """Sequential S6 scan, mlx_vision_mamba/mamba_block.py:20-74.

    x, delta: (B, L, D_inner); A: (D_inner, N); B, C: (B, L, N); D: (D_inner,).
    Returns y (B, L, D_inner) = sum_n h_t * C_t + x * D.
    """
    batch, seq_len, d_inner = x.shape
    n_state = A.shape[1]
    deltaA, deltaB_x = _discretize(x, delta, A, B)
    # unbind == per-step slicing, but lets autograd gather the step gradients
    # once instead of materialising a full-size zero gradient per step
    dA_t, dBx_t, C_t = deltaA.unbind(1), deltaB_x.unbind(1), C.unsqueeze(2).unbind(1)
    h = torch.zeros((batch, d_inner, n_state), dtype=x.dtype)
    ys = []
    for t in range(seq_len):                                   # mamba_block.py:64-68
        h = dA_t[t] * h + dBx_t[t]
        ys.append((h * C_t[t]).sum(dim=-1))
    y = torch.stack(ys, dim=1)
    return y + x * D                                           # mamba_block.py:73


def selective_scan_chunked(x, delta, A, B, C, D, chunk_size: int = 32):
    """Chunked variant, mlx_vision_mamba/mamba_fast.py:17-75 (same maths; the
    carry h crosses chunk boundaries)."""
    batch, seq_len, d_inner = x.shape
    n_state = A.shape[1]
    deltaA, deltaB_x = _discretize(x, delta, A, B)
    dA_t, dBx_t, C_t = deltaA.unbind(1), deltaB_x.unbind(1), C.unsqueeze(2).unbind(1)
    h = torch.zeros((batch, d_inner, n_state), dtype=x.dtype)
    outs = []
    for start in range(0, seq_len, chunk_size):                # mamba_fast.py:53-73
        stop = min(start + chunk_size, seq_len)
        ys = []
        for t in range(start, stop):
            h = dA_t[t] * h + dBx_t[t]
            ys.append((h * C_t[t]).sum(dim=-1))
        outs.append(torch.stack(ys, dim=1))
    y = torch.cat(outs, dim=1)
    return y + x * D


def silu(x):
    """MLX nn.silu: x * sigmoid(x)."""
    return x * torch.sigmoid(x)


def gated_scan(x, delta, A, B, C, D, z):
    """The scan followed by MambaBlock's gate y * silu(z) (mamba_block.py:187-190)."""
    return selective_scan(x, delta, A, B, C, D) * silu(z)


def sweep_inputs(batch, seq_len, d_inner, seed=0, dtype=torch.float32, d_state=16):
    """Seeded inputs of the op sweep: u, z ~ N(0,1); delta = softplus(0.5 N(0,1) - 3);
    A[d, n] = -(n+1); B, C ~ N(0,1); D = 1."""
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(batch, seq_len, d_inner, generator=g)
    z = torch.randn(batch, seq_len, d_inner, generator=g)
    delta = torch.nn.functional.softplus(0.5 * torch.randn(batch, seq_len, d_inner, generator=g) - 3.0)
    A = -torch.arange(1, d_state + 1, dtype=torch.float32).repeat(d_inner, 1)
    B = torch.randn(batch, seq_len, d_state, generator=g)
    C = torch.randn(batch, seq_len, d_state, generator=g)
    D = torch.ones(d_inner)
    dy = torch.randn(batch, seq_len, d_inner, generator=g)
    out = dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z, dy=dy)
    return {k: v.to(dtype) for k, v in out.items()}


def scan_vjp(inputs, gated=True, dtype=torch.float32, scan_fn=None):
    """Forward + VJP of the (optionally gated) scan via autograd; scan_fn is
    the sequential scan (default) or selective_scan_chunked.

    Returns (y, grads) with grads keyed du, ddelta, dA, dB, dC, dD[, dz].
    """
    scan_fn = scan_fn or selective_scan
    names = ["u", "delta", "A", "B", "C", "D"] + (["z"] if gated else [])
    leaves = {k: inputs[k].detach().to(dtype).clone().requires_grad_(True) for k in names}
    y = scan_fn(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"], leaves["D"])
    if gated:
        y = y * silu(leaves["z"])
    y.backward(inputs["dy"].to(dtype))
    grads = {"d" + k: leaves[k].grad.detach() for k in names}
    return y.detach(), grads
