"""VisionMamba encoder (2D / 3D / 4D) and its patch embeddings.

Mirror of mlx_vision_mamba/vision_mamba.py:25-228 and the patch embeddings of
mlx_vision_mamba/vit.py:48-92.  Inputs are channel-last as in MLX.  The patch
convolutions have stride == kernel size, so each is exactly a reshape of the
input into patches followed by one GEMM; their weights keep MLX's Conv layout
((E, p, p, C) for 2D, (E, p, p, p, C) for 3D) so MLX checkpoints load by name.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from .linear import linear_tc, supported as _tc_supported
from .mamba_block import LayerNorm, MultiDirectionalMambaBlock


def _patch_proj(x2: torch.Tensor, proj) -> torch.Tensor:
    """(N, patch features) @ W^T + b for a patch embedding: on the tensor-core
    GEMM (fp32 accuracy) when its operands qualify, else PyTorch's addmm."""
    wt = proj.weight.reshape(proj.weight.shape[0], -1)
    if _tc_supported(x2, wt):
        return linear_tc(x2, wt) + proj.bias
    return torch.addmm(proj.bias, x2, wt.t())


def _mlx_conv_init(weight: torch.Tensor, fan_in: int) -> None:
    with torch.no_grad():
        s = math.sqrt(1.0 / fan_in)
        weight.uniform_(-s, s)


class PatchEmbed(nn.Module):
    """(B, H, W, C) -> (B, H/p * W/p, E) (vit.py:48-67)."""

    def __init__(self, in_channels: int = 1, embed_dim: int = 384, patch_size: int = 16):
        super().__init__()
        self.patch_size = patch_size
        self.proj = nn.Module()
        self.proj.weight = nn.Parameter(torch.empty(embed_dim, patch_size, patch_size, in_channels))
        self.proj.bias = nn.Parameter(torch.zeros(embed_dim))
        _mlx_conv_init(self.proj.weight, in_channels * patch_size * patch_size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, h, w, c = x.shape
        p = self.patch_size
        hp, wp = h // p, w // p
        x = x[:, : hp * p, : wp * p, :].reshape(b, hp, p, wp, p, c).permute(0, 1, 3, 2, 4, 5)
        x = x.reshape(b, hp * wp, p * p * c)
        return _patch_proj(x.reshape(-1, x.shape[-1]), self.proj).reshape(b, hp * wp, -1)


class PatchEmbed3D(nn.Module):
    """(B, D, H, W, C) -> (B, D/p * H/p * W/p, E) (vit.py:70-92)."""

    def __init__(self, in_channels: int = 1, embed_dim: int = 384, patch_size: int = 16):
        super().__init__()
        self.patch_size = patch_size
        self.proj = nn.Module()
        self.proj.weight = nn.Parameter(torch.empty(embed_dim, patch_size, patch_size, patch_size, in_channels))
        self.proj.bias = nn.Parameter(torch.zeros(embed_dim))
        _mlx_conv_init(self.proj.weight, in_channels * patch_size ** 3)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, d, h, w, c = x.shape
        p = self.patch_size
        dp, hp, wp = d // p, h // p, w // p
        x = x[:, : dp * p, : hp * p, : wp * p, :].reshape(b, dp, p, hp, p, wp, p, c)
        x = x.permute(0, 1, 3, 5, 2, 4, 6, 7).reshape(b, dp * hp * wp, p * p * p * c)
        return _patch_proj(x.reshape(-1, x.shape[-1]), self.proj).reshape(b, dp * hp * wp, -1)


class PatchEmbed4D(nn.Module):
    """(B, T, D, H, W, C) -> (B, T/tp * D/p * H/p * W/p, E): temporal frames folded
    into channels, then the 3D embedding per frame group (vision_mamba.py:25-94)."""

    def __init__(self, in_channels: int = 1, embed_dim: int = 384, patch_size: int = 16,
                 temporal_patch_size: int = 1):
        super().__init__()
        self.patch_size = patch_size
        self.temporal_patch_size = temporal_patch_size
        self.proj = PatchEmbed3D(in_channels * temporal_patch_size, embed_dim, patch_size).proj

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, t, d, h, w, c = x.shape
        tp = self.temporal_patch_size
        if tp > 1:
            t_out = t // tp
            x = x[:, : t_out * tp].reshape(b, t_out, tp, d, h, w, c).permute(0, 1, 3, 4, 5, 2, 6)
            x = x.reshape(b, t_out, d, h, w, tp * c)
        else:
            t_out = t
        x = x.reshape(b * t_out, d, h, w, -1)
        p = self.patch_size
        dp, hp, wp = d // p, h // p, w // p
        cc = x.shape[-1]
        x = x[:, : dp * p, : hp * p, : wp * p, :].reshape(b * t_out, dp, p, hp, p, wp, p, cc)
        x = x.permute(0, 1, 3, 5, 2, 4, 6, 7).reshape(b * t_out * dp * hp * wp, p * p * p * cc)
        return _patch_proj(x, self.proj).reshape(b, t_out * dp * hp * wp, -1)


class VisionMamba(nn.Module):
    """PatchEmbed -> + pos_embed -> depth x MultiDirectionalMambaBlock -> LayerNorm
    (vision_mamba.py:97-228).  input_dim 2/3/4 selects K = 4/6/8 directions."""

    def __init__(
        self,
        img_size: int = 224,
        patch_size: int = 16,
        in_channels: int = 1,
        embed_dim: int = 384,
        depth: int = 6,
        d_state: int = 16,
        d_conv: int = 4,
        expand_factor: int = 2,
        input_dim: int = 2,
        temporal_patch_size: int = 1,
        num_temporal_frames: int = 1,
        scan_mode: str = "cuda_fused",
    ):
        super().__init__()
        self.embed_dim = embed_dim
        self.input_dim = input_dim
        self.img_size = img_size
        self.patch_size = patch_size
        g = img_size // patch_size
        if input_dim == 2:
            self.grid_shape = (g, g)
            self.num_patches = g * g
            num_directions = 4
            self.patch_embed = PatchEmbed(in_channels, embed_dim, patch_size)
        elif input_dim == 3:
            self.grid_shape = (g, g, g)
            self.num_patches = g ** 3
            num_directions = 6
            self.patch_embed = PatchEmbed3D(in_channels, embed_dim, patch_size)
        elif input_dim == 4:
            tg = num_temporal_frames // temporal_patch_size
            self.grid_shape = (tg, g, g, g)
            self.num_patches = tg * g ** 3
            num_directions = 8
            self.patch_embed = PatchEmbed4D(in_channels, embed_dim, patch_size, temporal_patch_size)
        else:
            raise ValueError(f"input_dim must be 2, 3, or 4, got {input_dim}")
        self.num_directions = num_directions
        self.pos_embed = nn.Parameter(torch.randn(1, self.num_patches, embed_dim) / math.sqrt(embed_dim))
        self.blocks = nn.ModuleList(
            [
                MultiDirectionalMambaBlock(
                    embed_dim, d_state, d_conv, expand_factor, num_directions=num_directions,
                    grid_shape=self.grid_shape, scan_mode=scan_mode,
                )
                for _ in range(depth)
            ]
        )
        self.norm = LayerNorm(embed_dim)

    def shard_directions(self, group) -> None:
        """Split every layer's scan directions across the ranks of `group`
        (MultiDirectionalMambaBlock.shard_directions); all ranks process the
        same batch."""
        for block in self.blocks:
            block.shard_directions(group)

    def forward(self, x: torch.Tensor, patch_indices: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x.dim() != 3:
            x = self.patch_embed(x)
        if patch_indices is not None:
            x = x + self.pos_embed[:, patch_indices, :]
        else:
            x = x + self.pos_embed
        for block in self.blocks:
            x = block(x)
        return self.norm(x)

    def embed_patches(self, images: torch.Tensor) -> torch.Tensor:
        return self.patch_embed(images)
