"""Mamba blocks for B200: the host-side mirror of mlx_vision_mamba/mamba_block.py.

Class names, constructor arguments, parameter names and parameter shapes follow
the reference (MLX layouts, e.g. conv1d.weight is (d_inner, d_conv, 1)), so an
MLX checkpoint's arrays load by name.  The selective scan, its SiLU gate and the
causal conv1d+SiLU run in the sm_100a kernels of libvmscan.so; in_proj and
out_proj run on its tensor-core GEMM (linear.py), x_proj on cuBLAS.  Multi-directional scans never build permuted copies: each
direction is a descriptor passed to the kernels (direction.py).

Deliberate deviations from the reference, all documented:
  * `scan_mode` defaults to "cuda_fused" and is threaded through every wrapper
    (the reference never forwards it, mamba_block.py:202,223-224,402-405).
  * The reference's Metal modes ("metal", "metal_train", "metal_fused") select
    the CUDA kernels; the CPU Python scans ("sequential", "chunked",
    "parallel") are not part of this package and unknown modes raise instead of
    silently falling back (mamba_block.py:121-122).
"""

from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .direction import BACKWARD, ScanDirection, directions_for
from .branches import block_core_forward, block_core_ok, branches_forward
from .linear import linear_tc, supported as _tc_supported
from .norm import layer_norm_cuda as _layer_norm_cuda, supported as _ln_supported
from .scan import conv1d_silu_cuda, dt_softplus_cuda, selective_scan_cuda

GPU_SCAN_MODES = ("cuda_fused", "metal_fused", "metal_train", "metal")
CPU_SCAN_MODES = ("sequential", "chunked", "parallel")


def _mlx_uniform_(t: torch.Tensor, scale: float) -> torch.Tensor:
    with torch.no_grad():
        return t.uniform_(-scale, scale)


class Linear(nn.Linear):
    """nn.Linear with MLX's default init: U(-1/sqrt(in), 1/sqrt(in)) for weight and bias."""

    def reset_parameters(self) -> None:
        scale = math.sqrt(1.0 / self.in_features)
        _mlx_uniform_(self.weight, scale)
        if self.bias is not None:
            _mlx_uniform_(self.bias, scale)


class LayerNorm(nn.LayerNorm):
    """MLX nn.LayerNorm defaults: eps 1e-5, weight 1, bias 0.

    CUDA fp32 inputs whose last dimension is a multiple of 4 and at most 1024
    (the encoders' 384) run forward and VJP in the library's LayerNorm kernels
    (`norm.layer_norm_cuda`); other inputs use PyTorch's layer_norm."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if len(self.normalized_shape) == 1 and _ln_supported(x, self.weight, self.bias):
            return _layer_norm_cuda(x, self.weight, self.bias, self.eps)
        return super().forward(x)


class DepthwiseConv1d(nn.Module):
    """Parameters of MLX's nn.Conv1d(C, C, K, padding=K-1, groups=C) in MLX layout.

    weight (C, K, 1) ~ U(-s, s) with s = sqrt(1 / (C * K)) and bias zeros, the
    MLX Conv1d initialisation.  The computation itself (causal, along the
    scan order, fused with SiLU) is `conv1d_silu_cuda`.
    """

    def __init__(self, channels: int, kernel_size: int):
        super().__init__()
        self.channels = channels
        self.kernel_size = kernel_size
        self.weight = nn.Parameter(torch.empty(channels, kernel_size, 1))
        self.bias = nn.Parameter(torch.zeros(channels))
        _mlx_uniform_(self.weight, math.sqrt(1.0 / (channels * kernel_size)))

    def silu_along(self, x: torch.Tensor, direction: Optional[ScanDirection]) -> torch.Tensor:
        return conv1d_silu_cuda(x, self.weight, self.bias, direction)


class MambaBlock(nn.Module):
    """in_proj -> causal depthwise conv1d -> SiLU -> x_proj -> dt_proj -> softplus
    -> selective scan -> y * SiLU(z) -> out_proj (mamba_block.py:77-192).

    `forward(x, direction=None)`: x is (B, L, d_model) in token order; with a
    direction the conv and the scan run along that order and the output comes
    back in token order, i.e. `unpermute(block(permute(x)))` of the reference
    without the copies.
    """

    def __init__(
        self,
        d_model: int = 384,
        d_state: int = 16,
        d_conv: int = 4,
        expand_factor: int = 2,
        scan_mode: str = "cuda_fused",
    ):
        super().__init__()
        if scan_mode in CPU_SCAN_MODES:
            raise ValueError(
                f"scan_mode={scan_mode!r} is a CPU Python scan of the reference; this package only "
                "implements the CUDA path (scan_mode='cuda_fused')"
            )
        if scan_mode not in GPU_SCAN_MODES:
            raise ValueError(f"unknown scan_mode {scan_mode!r}; expected one of {GPU_SCAN_MODES}")
        self.d_model = d_model
        self.d_state = d_state
        self.d_inner = d_model * expand_factor
        self.d_conv = d_conv
        self.scan_mode = scan_mode
        self.dt_rank = math.ceil(d_model / 16)

        self.in_proj = Linear(d_model, 2 * self.d_inner, bias=False)
        self.conv1d = DepthwiseConv1d(self.d_inner, d_conv)
        self.x_proj = Linear(self.d_inner, self.dt_rank + 2 * d_state, bias=False)
        self.dt_proj = Linear(self.dt_rank, self.d_inner, bias=True)
        a = torch.arange(1, d_state + 1, dtype=torch.float32).unsqueeze(0).repeat(self.d_inner, 1)
        self.A_log = nn.Parameter(torch.log(a))
        self.D = nn.Parameter(torch.ones(self.d_inner))
        self.out_proj = Linear(self.d_inner, d_model, bias=False)

    def forward(self, x: torch.Tensor, direction: Optional[ScanDirection] = None) -> torch.Tensor:
        if _fused_branches_ok([self], x) and block_core_ok([self], x):
            return block_core_forward([self], [direction], x, self.in_proj.weight, self.out_proj.weight,
                                      _branch_streams(x.device, 1))
        if _fused_branches_ok([self], x):
            xz = project(x, self.in_proj.weight)
            y = branches_forward([self], [direction], xz, _branch_streams(x.device, 1))
            return project(y, self.out_proj.weight)
        return project(self.scan_branch(project(x, self.in_proj.weight), direction), self.out_proj.weight)

    def scan_branch(self, xz: torch.Tensor, direction: Optional[ScanDirection] = None) -> torch.Tensor:
        """Everything between in_proj and out_proj (mamba_block.py:166-190): xz is
        the in_proj output (B, L, 2 d_inner), possibly a strided column slice of a
        wider projection; returns the gated scan output (B, L, d_inner)."""
        dn, r, n = self.d_inner, self.dt_rank, self.d_state
        # split (not slicing): its backward concatenates the pieces' gradients
        # instead of materialising a zero-filled full-width gradient per piece
        x_branch, z = torch.split(xz, [dn, dn], dim=-1)
        x_branch = self.conv1d.silu_along(x_branch, direction)
        x_dbc = self.x_proj(x_branch)
        dt, B_proj, C_proj = torch.split(x_dbc, [r, n, n], dim=-1)
        # dt_proj + bias + softplus (log(1 + exp(.)), mamba_block.py:180-181) in one kernel
        delta = dt_softplus_cuda(dt, self.dt_proj.weight, self.dt_proj.bias)
        A = -torch.exp(self.A_log)
        return selective_scan_cuda(x_branch, delta, A, B_proj, C_proj, self.D, z=z, direction=direction)


def project(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """x @ weight.T (in_proj / out_proj, no bias): on CUDA the fp32-accurate
    tensor-core GEMM of linear.py, elsewhere F.linear."""
    if _tc_supported(x, weight):
        return linear_tc(x, weight)
    return F.linear(x, weight)


def directions_sum(blocks: Sequence[MambaBlock], directions: Sequence[Optional[ScanDirection]], h: torch.Tensor):
    """sum_k blocks[k](h, directions[k]) with the projections batched over the
    directions: one in_proj GEMM against the K blocks' concatenated weights
    (each direction reads its column slice in place) and one out_proj GEMM over
    the concatenated inner dimension, which performs the sum over directions
    (the reference adds the K block outputs, mamba_block.py:562-566).  The
    parameters stay per block, as in the reference."""
    if len(blocks) == 1:
        return blocks[0](h, directions[0])
    two_dn = 2 * blocks[0].d_inner
    if _fused_branches_ok(blocks, h) and block_core_ok(blocks, h):
        # in_proj, the K branches and out_proj as one autograd node (branches.py)
        return block_core_forward(blocks, directions, h, torch.cat([b.in_proj.weight for b in blocks], 0),
                                  torch.cat([b.out_proj.weight for b in blocks], 1),
                                  _branch_streams(h.device, len(blocks)))
    xz = project(h, torch.cat([b.in_proj.weight for b in blocks], 0))
    if _fused_branches_ok(blocks, h):
        # one autograd node for the K branches: outputs and input gradients
        # written into slices, no concatenation passes (branches.py)
        y = branches_forward(blocks, directions, xz, _branch_streams(h.device, len(blocks)))
        return project(y, torch.cat([b.out_proj.weight for b in blocks], 1))
    parts = torch.split(xz, two_dn, dim=-1)
    if h.is_cuda:
        ys = _branches_on_streams(blocks, directions, parts)
    else:
        ys = [b.scan_branch(part, d) for b, d, part in zip(blocks, directions, parts)]
    return project(torch.cat(ys, -1), torch.cat([b.out_proj.weight for b in blocks], 1))


def _fused_branches_ok(blocks, h: torch.Tensor) -> bool:
    """The fused K-branch node applies to CUDA inputs of real MambaBlocks with
    one geometry and d_inner a multiple of 4 (its in-place x_proj gradient
    needs contiguous rows)."""
    if not h.is_cuda or not all(isinstance(b, MambaBlock) for b in blocks):
        return False
    b0 = blocks[0]
    same = all((b.d_inner, b.dt_rank, b.d_conv, b.d_state) == (b0.d_inner, b0.dt_rank, b0.d_conv, b0.d_state)
               for b in blocks)
    return same and b0.d_inner % 4 == 0 and b0.d_state == 16


_STREAMS = {}


def _branch_streams(device: torch.device, k: int):
    key = (device.index, k)
    if key not in _STREAMS:
        _STREAMS[key] = [torch.cuda.Stream(device=device) for _ in range(k)]
    return _STREAMS[key]


def _branches_on_streams(blocks, directions, parts):
    """Run the K independent direction branches (conv, x_proj, dt_proj, scan)
    concurrently, one CUDA stream each, so that small per-GPU batches still fill
    the GPU (a branch of batch 8 launches only a few dozen CTAs per kernel).
    Autograd runs each branch's backward on the same stream; under CUDA graph
    capture the streams become parallel branches of the graph."""
    cur = torch.cuda.current_stream(parts[0].device)
    streams = _branch_streams(parts[0].device, len(blocks))
    ys = []
    for b, d, part, s in zip(blocks, directions, parts, streams):
        s.wait_stream(cur)
        with torch.cuda.stream(s):
            ys.append(b.scan_branch(part, d))
    for y, s in zip(ys, streams):
        cur.wait_stream(s)
        y.record_stream(cur)
    return ys


class ResidualMambaBlock(nn.Module):
    """x + mamba(norm(x)) (mamba_block.py:195-205)."""

    def __init__(self, d_model=384, d_state=16, d_conv=4, expand_factor=2, scan_mode="cuda_fused"):
        super().__init__()
        self.norm = LayerNorm(d_model)
        self.mamba = MambaBlock(d_model, d_state, d_conv, expand_factor, scan_mode)

    def forward(self, x):
        return x + self.mamba(self.norm(x))


class BidirectionalMambaBlock(nn.Module):
    """x + fwd(norm(x)) + flip(bwd(flip(norm(x)))) (mamba_block.py:208-237); the flips
    are the BACKWARD direction of the kernels."""

    def __init__(self, d_model=384, d_state=16, d_conv=4, expand_factor=2, scan_mode="cuda_fused"):
        super().__init__()
        self.norm = LayerNorm(d_model)
        self.forward_mamba = MambaBlock(d_model, d_state, d_conv, expand_factor, scan_mode)
        self.backward_mamba = MambaBlock(d_model, d_state, d_conv, expand_factor, scan_mode)

    def forward(self, x):
        h = self.norm(x)
        return x + directions_sum([self.forward_mamba, self.backward_mamba], [None, BACKWARD], h)


class _ToDirectionRanks(torch.autograd.Function):
    """The block input entering the rank's direction branches: identity forward;
    backward all-reduces (sums) the branches' input gradients over the ranks."""

    @staticmethod
    def forward(ctx, h, group):
        ctx.group = group
        return h.view_as(h)

    @staticmethod
    def backward(ctx, grad):
        import torch.distributed as dist

        grad = grad.contiguous()
        dist.all_reduce(grad, group=ctx.group)
        return grad, None


class _FromDirectionRanks(torch.autograd.Function):
    """Sum of the directions over the ranks: all-reduce forward; identity
    backward (every rank holds the whole, replicated loss)."""

    @staticmethod
    def forward(ctx, y, group):
        import torch.distributed as dist

        y = y.contiguous().clone()
        dist.all_reduce(y, group=group)
        return y

    @staticmethod
    def backward(ctx, grad):
        return grad, None


class MultiDirectionalMambaBlock(nn.Module):
    """K independent MambaBlocks, one per scan direction, summed plus residual
    (mamba_block.py:341-566).  Directions follow `_apply_direction` (:407-534);
    when the sequence is not the full grid only blocks 0 and 1 run, forward and
    reversed (:550-559)."""

    def __init__(
        self,
        d_model: int = 384,
        d_state: int = 16,
        d_conv: int = 4,
        expand_factor: int = 2,
        num_directions: int = 2,
        grid_shape: Optional[Tuple[int, ...]] = None,
        scan_mode: str = "cuda_fused",
    ):
        super().__init__()
        if num_directions not in (2, 4, 6, 8):
            raise ValueError(f"num_directions must be 2, 4, 6, or 8, got {num_directions}")
        need = {4: 2, 6: 3, 8: 4}
        if num_directions > 2:
            if grid_shape is None:
                raise ValueError("grid_shape is required when num_directions > 2")
            if len(grid_shape) != need[num_directions]:
                raise ValueError(
                    f"K={num_directions} requires a {need[num_directions]}-D grid_shape, got {grid_shape}"
                )
        self.num_directions = num_directions
        self.grid_shape = tuple(grid_shape) if grid_shape is not None else None
        self.norm = LayerNorm(d_model)
        self.mamba_blocks = nn.ModuleList(
            [MambaBlock(d_model, d_state, d_conv, expand_factor, scan_mode) for _ in range(num_directions)]
        )
        self.directions = directions_for(num_directions, self.grid_shape)
        self.direction_group = None  # process group sharing the directions (shard_directions)

    def shard_directions(self, group) -> None:
        """Direction parallelism (no counterpart in the reference, which runs one
        device): rank r of `group` runs only the directions k with
        k % world == r and the partial sums are combined by an all-reduce whose
        backward sums the ranks' input gradients.  All ranks must feed the same
        input; every parameter keeps its reference name, and the parameters of
        the other ranks' directions simply receive no gradient here."""
        self.direction_group = group

    def _local(self, blocks, directions):
        import torch.distributed as dist

        world, rank = dist.get_world_size(self.direction_group), dist.get_rank(self.direction_group)
        ks = [k for k in range(len(blocks)) if k % world == rank]
        return [blocks[k] for k in ks], [directions[k] for k in ks]

    def _sum(self, blocks, directions, h):
        if self.direction_group is None:
            return directions_sum(blocks, directions, h)
        lb, ld = self._local(blocks, directions)
        hl = _ToDirectionRanks.apply(h, self.direction_group)
        y = directions_sum(lb, ld, hl) if lb else hl * 0.0
        return _FromDirectionRanks.apply(y, self.direction_group)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        n = x.shape[1]
        h = self.norm(x)
        expected = math.prod(self.grid_shape) if self.grid_shape is not None else n
        if n != expected and self.num_directions > 2:
            return x + self._sum(self.mamba_blocks[:2], [None, BACKWARD], h)
        return x + self._sum(self.mamba_blocks, self.directions, h)
