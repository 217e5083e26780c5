"""`mlx.nn` stand-in: the layers mlx-vision-mamba uses, on channel-last data.

Initialisations follow MLX's documented defaults: Linear weight and bias
U(-s, s) with s = 1/sqrt(in); ConvNd weight U(-s, s) with
s = 1/sqrt(in_channels * prod(kernel)), bias zero; LayerNorm weight 1, bias 0.
Weight layouts are MLX's: Linear (out, in); ConvNd (out, k..., in/groups).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import core as mx


class Module:
    def __init__(self):
        pass


class Linear(Module):
    def __init__(self, input_dims, output_dims, bias=True):
        s = math.sqrt(1.0 / input_dims)
        self.weight = mx.random.uniform(-s, s, (output_dims, input_dims))
        if bias:
            self.bias = mx.random.uniform(-s, s, (output_dims,))

    def __call__(self, x):
        y = x @ self.weight.transpose(0, 1)
        return mx._wrap(y + self.bias) if "bias" in vars(self) else mx._wrap(y)


def _tup(v, n):
    return tuple(v) if isinstance(v, (tuple, list)) else (v,) * n


class _ConvNd(Module):
    nd = 1

    def __init__(self, in_channels, out_channels, kernel_size, stride=1, padding=0, dilation=1, groups=1,
                 bias=True):
        k = _tup(kernel_size, self.nd)
        s = math.sqrt(1.0 / (in_channels * math.prod(k)))
        self.weight = mx.random.uniform(-s, s, (out_channels, *k, in_channels // groups))
        if bias:
            self.bias = mx.zeros((out_channels,))
        self.stride = _tup(stride, self.nd)
        self.padding = _tup(padding, self.nd)
        self.dilation = _tup(dilation, self.nd)
        self.groups = groups

    def __call__(self, x):
        nd = self.nd
        xc = x.permute(0, nd + 1, *range(1, nd + 1))
        w = self.weight.permute(0, nd + 1, *range(1, nd + 1))
        fn = {1: F.conv1d, 2: F.conv2d, 3: F.conv3d}[nd]
        y = fn(xc, w, self.bias if "bias" in vars(self) else None, stride=self.stride, padding=self.padding,
               dilation=self.dilation, groups=self.groups)
        return mx._wrap(y.permute(0, *range(2, nd + 2), 1))


class Conv1d(_ConvNd):
    nd = 1


class Conv2d(_ConvNd):
    nd = 2


class Conv3d(_ConvNd):
    nd = 3


class LayerNorm(Module):
    def __init__(self, dims, eps=1e-5, affine=True, bias=True):
        self.eps = eps
        self.dims = dims
        if affine:
            self.weight = mx.ones((dims,))
            if bias:
                self.bias = mx.zeros((dims,))

    def __call__(self, x):
        w = vars(self).get("weight")
        b = vars(self).get("bias")
        return mx._wrap(F.layer_norm(x, (self.dims,), w, b, self.eps))


def silu(x):
    return mx._wrap(x * torch.sigmoid(x))


def gelu(x):
    return mx._wrap(F.gelu(x))


class MultiHeadAttention(Module):
    def __init__(self, *a, **k):
        raise NotImplementedError("not needed for the selective-scan fixtures")
