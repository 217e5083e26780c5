"""`mlx.core` stand-in: arrays are torch tensors of the `array` subclass below."""

from __future__ import annotations

import torch

float32 = torch.float32
float64 = torch.float64
_DEFAULT = {"dtype": torch.float32}


def set_default_dtype(dt):
    """Fixture helper (not MLX): dtype of arrays created by zeros/ones/arange/random."""
    _DEFAULT["dtype"] = dt


class array(torch.Tensor):
    """torch.Tensor whose indexing also accepts MLX/numpy-style `::-1` slices."""

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func is torch.Tensor.__getitem__:
            t, idx = args
            items = idx if isinstance(idx, tuple) else (idx,)
            if any(isinstance(it, slice) and it.step is not None and it.step < 0 for it in items):
                with torch._C.DisableTorchFunctionSubclass():
                    dim = 0
                    clean = []
                    for it in items:
                        if isinstance(it, slice) and it.step is not None and it.step < 0:
                            if it.step != -1 or it.start is not None or it.stop is not None:
                                raise NotImplementedError("only [::-1] reversal is supported")
                            t = torch.flip(t, dims=[dim])
                            clean.append(slice(None))
                            dim += 1
                        elif it is None:
                            clean.append(it)
                        elif isinstance(it, int):
                            clean.append(it)
                        else:
                            clean.append(it)
                            dim += 1
                    out = t[tuple(clean)]
                return out.as_subclass(cls)
        return super().__torch_function__(func, types, args, kwargs)

    def astype(self, dtype):
        return self.to(dtype)


def _wrap(t):
    return t.as_subclass(array) if not isinstance(t, array) else t


def asarray(x, dtype=None):
    return _wrap(torch.as_tensor(x, dtype=dtype if dtype is not None else _DEFAULT["dtype"]))


def expand_dims(a, axis):
    return _wrap(torch.unsqueeze(a, axis))


def exp(a):
    return _wrap(torch.exp(a))


def log(a):
    return _wrap(torch.log(a))


def zeros(shape, dtype=None):
    return _wrap(torch.zeros(shape, dtype=dtype or _DEFAULT["dtype"]))


def ones(shape, dtype=None):
    return _wrap(torch.ones(shape, dtype=dtype or _DEFAULT["dtype"]))


def zeros_like(a):
    return _wrap(torch.zeros_like(a))


def stack(arrays, axis=0):
    return _wrap(torch.stack(list(arrays), dim=axis))


def concatenate(arrays, axis=0):
    return _wrap(torch.cat(list(arrays), dim=axis))


def repeat(a, repeats, axis=None):
    if axis is None:
        return _wrap(torch.repeat_interleave(a.reshape(-1), repeats))
    return _wrap(torch.repeat_interleave(a, repeats, dim=axis))


def arange(start, stop=None, step=1, dtype=None):
    if stop is None:
        start, stop = 0, start
    dt = dtype or _DEFAULT["dtype"]
    return _wrap(torch.arange(start, stop, step, dtype=dt))


def transpose(a, axes=None):
    if axes is None:
        axes = tuple(range(a.dim() - 1, -1, -1))
    return _wrap(a.permute(*axes))


def contiguous(a):
    return _wrap(a.contiguous())


def eval(*args):  # MLX is lazy; torch is eager
    return None


class _Random:
    generator = torch.Generator().manual_seed(0)

    def seed(self, s):
        self.generator = torch.Generator().manual_seed(int(s))

    def normal(self, shape=(), dtype=None, loc=0.0, scale=1.0):
        t = torch.randn(tuple(shape), generator=self.generator, dtype=torch.float64)
        return _wrap((t * scale + loc).to(dtype or _DEFAULT["dtype"]))

    def uniform(self, low=0.0, high=1.0, shape=(), dtype=None):
        t = torch.rand(tuple(shape), generator=self.generator, dtype=torch.float64)
        return _wrap((low + (high - low) * t).to(dtype or _DEFAULT["dtype"]))


random = _Random()


class _Fast:
    @staticmethod
    def metal_kernel(*args, **kwargs):
        raise RuntimeError("Metal kernels cannot run outside Apple GPUs")


fast = _Fast()


class custom_function:
    """Decorator stand-in: calls the primal; `.vjp` only registers (unused here)."""

    def __init__(self, fn):
        self.fn = fn
        self.vjp_fn = None

    def __call__(self, *args, **kwargs):
        return self.fn(*args, **kwargs)

    def vjp(self, fn):
        self.vjp_fn = fn
        return fn
