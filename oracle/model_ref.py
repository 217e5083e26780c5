"""CPU oracle of the blocks and the encoder around the scan.

TEST INFRASTRUCTURE ONLY.  Restates, on the CPU with torch:
  MambaBlock.__call__             mlx_vision_mamba/mamba_block.py:155-192
  ResidualMambaBlock              :195-205
  BidirectionalMambaBlock         :208-237
  permutation helpers             :244-338
  MultiDirectionalMambaBlock      :341-566 (direction table :407-534)
  PatchEmbed / PatchEmbed3D       mlx_vision_mamba/vit.py:48-92
  PatchEmbed4D / VisionMamba      mlx_vision_mamba/vision_mamba.py:25-228
Unlike the product, it keeps the reference's data movement literally: the
sequence is permuted and flipped, the block runs, the result is flipped and
un-permuted.  The MLX layers are restated with torch.nn.functional (conv on
channel-last data via transposes; MLX Conv weight layouts (out, k..., in)).
Parameter names and shapes equal the product's, so state dicts are shared.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .scan_ref import selective_scan, silu


class _Linear(nn.Module):
    def __init__(self, din, dout, bias):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(dout, din))
        self.bias = nn.Parameter(torch.empty(dout)) if bias else None
        s = math.sqrt(1.0 / din)
        with torch.no_grad():
            self.weight.uniform_(-s, s)
            if self.bias is not None:
                self.bias.uniform_(-s, s)

    def forward(self, x):
        y = x @ self.weight.t()
        return y + self.bias if self.bias is not None else y


class _LayerNorm(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.bias = nn.Parameter(torch.zeros(d))

    def forward(self, x):
        return F.layer_norm(x, (x.shape[-1],), self.weight, self.bias, eps=1e-5)


class _Conv1d(nn.Module):
    """MLX nn.Conv1d(C, C, K, padding=K-1, groups=C) on channel-last input."""

    def __init__(self, c, k):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(c, k, 1))
        self.bias = nn.Parameter(torch.zeros(c))
        s = math.sqrt(1.0 / (c * k))
        with torch.no_grad():
            self.weight.uniform_(-s, s)

    def forward(self, x):
        c, k = self.weight.shape[0], self.weight.shape[1]
        w = self.weight.permute(0, 2, 1)  # (C, 1, K)
        y = F.conv1d(x.transpose(1, 2), w, self.bias, padding=k - 1, groups=c)
        return y.transpose(1, 2)  # (B, L + K - 1, C)


class MambaBlockRef(nn.Module):
    def __init__(self, d_model=384, d_state=16, d_conv=4, expand_factor=2):
        super().__init__()
        self.d_model = d_model
        self.d_state = d_state
        self.d_inner = d_model * expand_factor
        self.d_conv = d_conv
        self.dt_rank = math.ceil(d_model / 16)
        self.in_proj = _Linear(d_model, 2 * self.d_inner, False)
        self.conv1d = _Conv1d(self.d_inner, d_conv)
        self.x_proj = _Linear(self.d_inner, self.dt_rank + 2 * d_state, False)
        self.dt_proj = _Linear(self.dt_rank, self.d_inner, True)
        a = torch.arange(1, d_state + 1, dtype=torch.float32).unsqueeze(0).repeat(self.d_inner, 1)
        self.A_log = nn.Parameter(torch.log(a))
        self.D = nn.Parameter(torch.ones(self.d_inner))
        self.out_proj = _Linear(self.d_inner, d_model, False)

    def forward(self, x):
        B, L, _ = x.shape
        dn, r, n = self.d_inner, self.dt_rank, self.d_state
        xz = self.in_proj(x)
        x_branch = xz[:, :, :dn]
        z = xz[:, :, dn:]
        x_branch = self.conv1d(x_branch)[:, :L, :]
        x_branch = silu(x_branch)
        x_dbc = self.x_proj(x_branch)
        dt = x_dbc[:, :, :r]
        B_proj = x_dbc[:, :, r : r + n]
        C_proj = x_dbc[:, :, r + n :]
        delta = self.dt_proj(dt)
        delta = torch.log(1.0 + torch.exp(delta))
        A = -torch.exp(self.A_log)
        y = selective_scan(x_branch, delta, A, B_proj, C_proj, self.D)
        y = y * silu(z)
        return self.out_proj(y)


class ResidualMambaBlockRef(nn.Module):
    def __init__(self, d_model=384, d_state=16, d_conv=4, expand_factor=2):
        super().__init__()
        self.norm = _LayerNorm(d_model)
        self.mamba = MambaBlockRef(d_model, d_state, d_conv, expand_factor)

    def forward(self, x):
        return x + self.mamba(self.norm(x))


def _flip(h):
    return torch.flip(h, dims=[1])


class BidirectionalMambaBlockRef(nn.Module):
    def __init__(self, d_model=384, d_state=16, d_conv=4, expand_factor=2):
        super().__init__()
        self.norm = _LayerNorm(d_model)
        self.forward_mamba = MambaBlockRef(d_model, d_state, d_conv, expand_factor)
        self.backward_mamba = MambaBlockRef(d_model, d_state, d_conv, expand_factor)

    def forward(self, x):
        h = self.norm(x)
        return x + self.forward_mamba(h) + _flip(self.backward_mamba(_flip(h)))


# permutation helpers, mamba_block.py:244-338
def permute_2d_col_major(h, grid):
    B, N, D = h.shape
    H, W = grid
    return h.reshape(B, H, W, D).permute(0, 2, 1, 3).reshape(B, N, D)


def unpermute_2d_col_major(h, grid):
    B, N, D = h.shape
    H, W = grid
    return h.reshape(B, W, H, D).permute(0, 2, 1, 3).reshape(B, N, D)


def permute_axes(h, grid, axes):
    B, N, D = h.shape
    nd = len(grid)
    h = h.reshape(B, *grid, D)
    perm = (0,) + tuple(a + 1 for a in axes) + (nd + 1,)
    return h.permute(*perm).reshape(B, N, D)


def unpermute_axes(h, grid, axes):
    B, N, D = h.shape
    nd = len(grid)
    h = h.reshape(B, *(grid[a] for a in axes), D)
    inv = [0] * nd
    for i, a in enumerate(axes):
        inv[a] = i
    perm = (0,) + tuple(a + 1 for a in inv) + (nd + 1,)
    return h.permute(*perm).reshape(B, N, D)


_AXIS_PERMS = {
    6: [(0, 1, 2), (1, 0, 2), (2, 0, 1)],
    8: [(0, 1, 2, 3), (1, 0, 2, 3), (2, 0, 1, 3), (3, 0, 1, 2)],
}


class MultiDirectionalMambaBlockRef(nn.Module):
    def __init__(self, d_model=384, d_state=16, d_conv=4, expand_factor=2, num_directions=2,
                 grid_shape: Optional[Tuple[int, ...]] = None):
        super().__init__()
        self.num_directions = num_directions
        self.grid_shape = tuple(grid_shape) if grid_shape is not None else None
        self.norm = _LayerNorm(d_model)
        self.mamba_blocks = nn.ModuleList(
            [MambaBlockRef(d_model, d_state, d_conv, expand_factor) for _ in range(num_directions)]
        )

    def apply_direction(self, h, k):
        """mamba_block.py:407-534."""
        mamba = self.mamba_blocks[k]
        K = self.num_directions
        rev = k % 2 == 1
        if K == 2:
            return _flip(mamba(_flip(h))) if rev else mamba(h)
        pair = k // 2
        if K == 4:
            if pair == 0:
                seq = _flip(h) if rev else h
                out = mamba(seq)
                return _flip(out) if rev else out
            seq = permute_2d_col_major(h, self.grid_shape)
            seq = _flip(seq) if rev else seq
            out = mamba(seq)
            out = _flip(out) if rev else out
            return unpermute_2d_col_major(out, self.grid_shape)
        perm = _AXIS_PERMS[K][pair]
        if perm == tuple(range(len(perm))):
            seq = _flip(h) if rev else h
            out = mamba(seq)
            return _flip(out) if rev else out
        seq = permute_axes(h, self.grid_shape, perm)
        seq = _flip(seq) if rev else seq
        out = mamba(seq)
        out = _flip(out) if rev else out
        return unpermute_axes(out, self.grid_shape, perm)

    def forward(self, x):
        B, N, D = x.shape
        h = self.norm(x)
        expected = math.prod(self.grid_shape) if self.grid_shape is not None else N
        if N != expected and self.num_directions > 2:
            y_fwd = self.mamba_blocks[0](h)
            y_bwd = _flip(self.mamba_blocks[1](_flip(h)))
            return x + y_fwd + y_bwd
        y = self.apply_direction(h, 0)
        for k in range(1, self.num_directions):
            y = y + self.apply_direction(h, k)
        return x + y


class _ConvNd(nn.Module):
    """MLX ConvNd with stride == kernel on channel-last input; weight (E, p.., C)."""

    def __init__(self, cin, e, p, nd):
        super().__init__()
        self.nd = nd
        self.p = p
        self.weight = nn.Parameter(torch.empty(e, *([p] * nd), cin))
        self.bias = nn.Parameter(torch.zeros(e))
        s = math.sqrt(1.0 / (cin * p ** nd))
        with torch.no_grad():
            self.weight.uniform_(-s, s)

    def forward(self, x):
        nd = self.nd
        xc = x.permute(0, nd + 1, *range(1, nd + 1))               # to channels-first
        w = self.weight.permute(0, nd + 1, *range(1, nd + 1))
        conv = F.conv2d if nd == 2 else F.conv3d
        y = conv(xc, w, self.bias, stride=self.p)
        return y.permute(0, *range(2, nd + 2), 1)                  # back to channel-last


class PatchEmbedRef(nn.Module):
    def __init__(self, in_channels=1, embed_dim=384, patch_size=16, nd=2):
        super().__init__()
        self.proj = _ConvNd(in_channels, embed_dim, patch_size, nd)

    def forward(self, x):
        y = self.proj(x)
        return y.reshape(y.shape[0], -1, y.shape[-1])


class PatchEmbed4DRef(nn.Module):
    def __init__(self, in_channels=1, embed_dim=384, patch_size=16, temporal_patch_size=1):
        super().__init__()
        self.tp = temporal_patch_size
        self.proj = _ConvNd(in_channels * temporal_patch_size, embed_dim, patch_size, 3)

    def forward(self, x):
        B, T, D, H, W, C = x.shape
        tp = self.tp
        if tp > 1:
            T_out = T // tp
            x = x.reshape(B, T_out, tp, D, H, W, C).permute(0, 1, 3, 4, 5, 2, 6).reshape(B, T_out, D, H, W, tp * C)
        else:
            T_out = T
        x = x.reshape(B * T_out, D, H, W, -1)
        y = self.proj(x)
        _, Dp, Hp, Wp, E = y.shape
        return y.reshape(B, T_out * Dp * Hp * Wp, E)


class VisionMambaRef(nn.Module):
    def __init__(self, img_size=224, patch_size=16, in_channels=1, embed_dim=384, depth=6, d_state=16,
                 d_conv=4, expand_factor=2, input_dim=2, temporal_patch_size=1, num_temporal_frames=1):
        super().__init__()
        g = img_size // patch_size
        if input_dim == 2:
            self.grid_shape = (g, g)
            K = 4
            self.patch_embed = PatchEmbedRef(in_channels, embed_dim, patch_size, 2)
        elif input_dim == 3:
            self.grid_shape = (g, g, g)
            K = 6
            self.patch_embed = PatchEmbedRef(in_channels, embed_dim, patch_size, 3)
        elif input_dim == 4:
            self.grid_shape = (num_temporal_frames // temporal_patch_size, g, g, g)
            K = 8
            self.patch_embed = PatchEmbed4DRef(in_channels, embed_dim, patch_size, temporal_patch_size)
        else:
            raise ValueError(input_dim)
        self.num_patches = math.prod(self.grid_shape)
        self.pos_embed = nn.Parameter(torch.randn(1, self.num_patches, embed_dim) / math.sqrt(embed_dim))
        self.blocks = nn.ModuleList(
            [MultiDirectionalMambaBlockRef(embed_dim, d_state, d_conv, expand_factor, K, self.grid_shape)
             for _ in range(depth)]
        )
        self.norm = _LayerNorm(embed_dim)

    def forward(self, x, patch_indices=None):
        if x.dim() != 3:
            x = self.patch_embed(x)
        x = x + (self.pos_embed[:, patch_indices, :] if patch_indices is not None else self.pos_embed)
        for blk in self.blocks:
            x = blk(x)
        return self.norm(x)
