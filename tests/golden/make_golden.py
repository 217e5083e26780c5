"""Generate golden fixtures by running the reference's own Python source.

    python tests/golden/make_golden.py --reference <path to an mlx-vision-mamba checkout>

The reference needs Apple MLX, which is not available on Linux.  This script
puts `tests/golden/mlx_shim` (a torch-backed stand-in for the MLX primitives
the reference calls) first on sys.path, imports the reference package from
the given checkout (read-only, nothing is copied) and runs its code:
`selective_scan`, `selective_scan_chunked`, `MambaBlock`,
`BidirectionalMambaBlock`, `MultiDirectionalMambaBlock` (K = 2/4/6/8 and the
subset fallback) and `VisionMamba` (2D/3D/4D).  Gradients come from torch
autograd through the reference code.  Each case is saved as a small .pt file
of inputs, parameters (by MLX name), outputs and gradients, in fp32.

The fixtures pin the CPU oracle (tests/test_oracle_golden.py) and the CUDA
path (the fixture cases of tests/test_scan_gpu.py and tests/test_block_gpu.py)
to the reference's behaviour, including its direction permutations and
operation order.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(ref_root: str):
    sys.path.insert(0, os.path.join(HERE, "mlx_shim"))
    sys.path.insert(0, ref_root)
    import mlx.core as mx  # noqa: F401  (the shim)
    import mlx_vision_mamba as ref

    return ref


def _named_arrays(obj, prefix=""):
    """Walk an MLX-style module: array attributes and sub-modules (incl. lists)."""
    import mlx.nn as nn

    out = {}
    for k, v in vars(obj).items():
        name = f"{prefix}{k}"
        if isinstance(v, torch.Tensor):
            out[name] = v
        elif isinstance(v, nn.Module):
            out.update(_named_arrays(v, name + "."))
        elif isinstance(v, (list, tuple)) and v and all(isinstance(m, nn.Module) for m in v):
            for i, m in enumerate(v):
                out.update(_named_arrays(m, f"{name}.{i}."))
    return out


def _set_arrays(obj, values, prefix=""):
    import mlx.nn as nn

    for k, v in list(vars(obj).items()):
        name = f"{prefix}{k}"
        if isinstance(v, torch.Tensor) and name in values:
            setattr(obj, k, values[name])
        elif isinstance(v, nn.Module):
            _set_arrays(v, values, name + ".")
        elif isinstance(v, (list, tuple)) and v and all(isinstance(m, nn.Module) for m in v):
            for i, m in enumerate(v):
                _set_arrays(m, values, f"{name}.{i}.")


def _leafify(module):
    """Make every parameter a fresh leaf requiring grad; return name -> leaf."""
    import mlx.core as mx

    arrs = _named_arrays(module)
    leaves = {k: mx._wrap(v.detach().clone()).requires_grad_(True) for k, v in arrs.items()}
    _set_arrays(module, leaves)
    return leaves


def _plain(t):
    return t.detach().as_subclass(torch.Tensor).clone().contiguous()


def _sweep_inputs(b, l, dn, seed, random_A=False):
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(b, l, dn, generator=g)
    z = torch.randn(b, l, dn, generator=g)
    delta = torch.nn.functional.softplus(0.5 * torch.randn(b, l, dn, generator=g) - 3.0)
    if random_A:
        A = -torch.exp(0.5 * torch.randn(dn, 16, generator=g))
    else:
        A = -torch.arange(1, 17, dtype=torch.float32).repeat(dn, 1)
    B = torch.randn(b, l, 16, generator=g)
    C = torch.randn(b, l, 16, generator=g)
    D = 1.0 + 0.1 * torch.randn(dn, generator=g)
    dy = torch.randn(b, l, dn, generator=g)
    return dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z, dy=dy)


def scan_case(ref, name, b, l, dn, seed, random_A=False, gated=True):
    import mlx.core as mx
    import mlx.nn as nn

    inp = _sweep_inputs(b, l, dn, seed, random_A)
    keys = ["u", "delta", "A", "B", "C", "D"] + (["z"] if gated else [])
    lv = {k: mx._wrap(inp[k].clone()).requires_grad_(True) for k in keys}
    y = ref.selective_scan(lv["u"], lv["delta"], lv["A"], lv["B"], lv["C"], lv["D"])
    if gated:
        y = y * nn.silu(lv["z"])
    (y * inp["dy"]).sum().backward()
    rec = {"inputs": {k: v.clone() for k, v in inp.items()}, "gated": gated, "y": _plain(y),
           "grads": {"d" + k: _plain(lv[k].grad) for k in keys}}
    from mlx_vision_mamba.mamba_fast import selective_scan_chunked

    rec["y_chunked"] = _plain(selective_scan_chunked(*(mx._wrap(inp[k]) for k in keys[:6])))
    return name, rec


def module_case(name, module, x, seed, call=None):
    leaves = _leafify(module)
    g = torch.Generator().manual_seed(seed + 1)
    xin = x.clone().requires_grad_(True)
    import mlx.core as mx

    xw = mx._wrap(xin)
    y = call(module, xw) if call else module(xw)
    dy = torch.randn(y.shape, generator=g)
    (y * dy).sum().backward()
    return name, {
        "x": x.clone(),
        "dy": dy,
        "y": _plain(y),
        "dx": _plain(xin.grad),
        "params": {k: _plain(v) for k, v in leaves.items()},
        "grads": {k: _plain(v.grad) if v.grad is not None else torch.zeros_like(_plain(v)) for k, v in leaves.items()},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout root of mlx-vision-mamba")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    ref = _import_reference(args.reference)
    import mlx.core as mx

    torch.manual_seed(0)
    mx.random.seed(0)
    cases = []
    # selective_scan: ragged and multi-box lengths, channel counts not multiple of the tile
    cases.append(scan_case(ref, "scan_b2_l7_d8", 2, 7, 8, 1))
    cases.append(scan_case(ref, "scan_b1_l33_d12_randA", 1, 33, 12, 2, random_A=True))
    cases.append(scan_case(ref, "scan_b2_l40_d40_plain", 2, 40, 40, 3, gated=False))
    cases.append(scan_case(ref, "scan_b1_l1_d4", 1, 1, 4, 4))

    def x_of(shape, seed):
        return torch.randn(*shape, generator=torch.Generator().manual_seed(seed))

    mx.random.seed(10)
    cases.append(module_case("mamba_block_d16_l10", ref.MambaBlock(16, 16, 4, 2), x_of((2, 10, 16), 11), 11))
    mx.random.seed(12)
    cases.append(module_case("bidir_d8_l9", ref.BidirectionalMambaBlock(8, 16, 4, 2), x_of((2, 9, 8), 12), 12))
    for K, grid, seed in ((2, (12,), 20), (4, (3, 4), 21), (6, (2, 3, 2), 22), (8, (2, 2, 3, 2), 23)):
        mx.random.seed(seed)
        blk = ref.MultiDirectionalMambaBlock(8, 16, 4, 2, num_directions=K, grid_shape=grid)
        n = 1
        for gdim in grid:
            n *= gdim
        cases.append(module_case(f"multidir_k{K}", blk, x_of((2, n, 8), seed), seed))
    mx.random.seed(24)
    blk = ref.MultiDirectionalMambaBlock(8, 16, 4, 2, num_directions=4, grid_shape=(3, 4))
    cases.append(module_case("multidir_k4_subset", blk, x_of((1, 7, 8), 24), 24))
    for dim, kw, shape, seed in (
        (2, {}, (2, 8, 8, 1), 30),
        (3, {}, (1, 8, 8, 8, 1), 31),
        (4, {"num_temporal_frames": 2}, (1, 2, 8, 8, 8, 1), 32),
    ):
        mx.random.seed(seed)
        vm = ref.VisionMamba(img_size=8, patch_size=4, in_channels=1, embed_dim=8, depth=1, input_dim=dim, **kw)
        cases.append(module_case(f"vision_mamba_{dim}d", vm, x_of(shape, seed), seed))

    os.makedirs(args.out, exist_ok=True)
    total = 0
    for name, rec in cases:
        path = os.path.join(args.out, name + ".pt")
        torch.save(rec, path)
        total += os.path.getsize(path)
        print(f"wrote {path}")
    print(f"{len(cases)} fixtures, {total / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
