"""Parity rule shared by the GPU tests.

The north-star tolerance is 1e-5 relative / 1e-6 absolute on fp32 outputs and
gradients.  It is measured against the exact result of the reference
algorithm (the oracle in fp64), and the reference's own fp32 result (`ref32`,
the oracle in fp32 or a fixture produced by the reference's source) is
measured the same way.

The reference's fp32 arithmetic does not meet 1e-5/1e-6 everywhere: ddelta
sums A[n] * g[n] (|A| up to 16) against u * sum(dh * B) and cancels, and dw /
dbias of the conv sum hundreds of signed terms.  At such elements no fp32
implementation with another summation order can stay within 1e-5/1e-6 of the
reference.  The rule is therefore, per output tensor:

  element-wise  |ours - exact| <= ATOL + RTOL * |exact| + 2 * max|ref32 - exact|
                (no element worse than twice the reference's own worst error
                on that tensor, on top of the north-star bound), and
  norm-wise     ||ours - exact||_2 <= 2 * ||ref32 - exact||_2 + ATOL * sqrt(n)
                (on average no less accurate than half the reference's accuracy).

Without a ref32 the element-wise rule is the plain north-star bound.  The
fraction of elements inside the plain bound is reported on failure.
"""

import math

import torch

from conftest import ATOL, RTOL

# One row per checked tensor, written out as a table at the end of the
# session when VMSCAN_PARITY_TABLE names a file (tests/conftest.py):
#   name, n (elements), strict (fraction of ours within the plain
#   1e-5 / 1e-6 bound of the exact result), ref32_strict (the same fraction for
#   the reference's fp32 result), ratio (worst element error / enforced
#   bound), vs_ref32 (max |ours - ref32| / (1e-6 + 1e-5 |ref32|)).
RECORDS = []


def parity_report(ours, ref64, ref32=None, rtol=RTOL, atol=ATOL, name=None):
    ours = ours.detach().double().cpu()
    ref64 = ref64.detach().double().cpu()
    err = (ours - ref64).abs()
    strict_bound = atol + rtol * ref64.abs()
    bound = strict_bound
    norm_ok = True
    norm_ratio = 0.0
    ref_strict = None
    vs_ref32 = None
    if ref32 is not None:
        r32 = ref32.detach().double().cpu()
        ref_err = (r32 - ref64).abs()
        bound = strict_bound + 2.0 * (ref_err.max() if ref_err.numel() else 0.0)
        lhs = err.norm().item()
        rhs = 2.0 * ref_err.norm().item() + atol * math.sqrt(max(err.numel(), 1))
        norm_ratio = lhs / rhs
        norm_ok = lhs <= rhs
        if ref_err.numel():
            ref_strict = (ref_err <= strict_bound).double().mean().item()
            vs_ref32 = ((ours - r32).abs() / (atol + rtol * r32.abs())).max().item()
    ratio = (err / bound).max().item() if err.numel() else 0.0
    strict = (err <= strict_bound).double().mean().item() if err.numel() else 1.0
    if name is not None:
        RECORDS.append({"name": name, "n": int(err.numel()), "strict": strict, "ref32_strict": ref_strict,
                        "ratio": ratio, "norm_ratio": norm_ratio if ref32 is not None else None,
                        "vs_ref32": vs_ref32})
    return ratio, strict, norm_ok, norm_ratio


def assert_parity(name, ours, ref64, ref32=None, rtol=RTOL, atol=ATOL):
    assert ours.shape == ref64.shape, (name, tuple(ours.shape), tuple(ref64.shape))
    assert torch.isfinite(ours).all(), f"{name}: non-finite values"
    ratio, strict, norm_ok, norm_ratio = parity_report(ours, ref64, ref32, rtol, atol, name=name)
    assert ratio <= 1.0 and norm_ok, (
        f"{name}: element error/bound = {ratio:.3f}, norm error ratio = {norm_ratio:.3f} "
        f"(fraction within plain 1e-5/1e-6: {strict:.6f})"
    )


# bf16 I/O: an fp32 result rounded to bf16 (8 significand bits, round to
# nearest even) is off by at most 2^-8 of its magnitude on top of the fp32
# error.
BF16_ROUND = 2.0**-8


def assert_parity_bf16(name, ours, ref64, ref32=None):
    """Parity of a bf16 output computed in fp32 and rounded once at the store.

    element-wise  |ours - exact| <= (fp32 bound of assert_parity) + 2^-8 |exact|
    norm-wise     ||ours - exact||_2 <= 2 ||bf16(exact) - exact||_2
                                        + 2 ||ref32 - exact||_2 + ATOL sqrt(n)
                  (on average no less accurate than half the accuracy of
                  rounding the exact result to bf16).
    """
    ours = ours.detach().double().cpu()
    ref64 = ref64.detach().double().cpu()
    assert ours.shape == ref64.shape, (name, tuple(ours.shape), tuple(ref64.shape))
    assert torch.isfinite(ours).all(), f"{name}: non-finite values"
    err = (ours - ref64).abs()
    bound = ATOL + (RTOL + BF16_ROUND) * ref64.abs()
    rhs = 2.0 * (ref64.to(torch.bfloat16).double() - ref64).norm().item() + ATOL * math.sqrt(max(err.numel(), 1))
    if ref32 is not None:
        ref_err = (ref32.detach().double().cpu() - ref64).abs()
        bound = bound + 2.0 * (ref_err.max() if ref_err.numel() else 0.0)
        rhs += 2.0 * ref_err.norm().item()
    ratio = (err / bound).max().item() if err.numel() else 0.0
    lhs = err.norm().item()
    assert ratio <= 1.0 and lhs <= rhs, f"{name}: element error/bound = {ratio:.3f}, norm error ratio = {lhs / rhs:.3f}"


def oracle_vjp(inputs, dtype, split=None, piece=256):
    """scan_ref.scan_vjp (gated) on `inputs`, optionally in independent pieces.

    split="channels": pieces of `piece` channels (the recurrence never crosses
    channels); y, du, ddelta, dz, dA, dD are concatenated and dB, dC summed
    over the pieces.  split="batch": pieces of `piece` batch rows; dA, dD are
    summed.  Summing pieces in fp64 is exact to far below the tolerances; the
    pieces keep every temporary small, which on the CPU is several times
    faster than one call (the large (B, L, D, N) temporaries of one call are
    dominated by page faults)."""
    from oracle import scan_ref

    if split is None:
        return scan_ref.scan_vjp(inputs, gated=True, dtype=dtype)
    seq = ("u", "z", "delta", "dy")
    if split == "channels":
        n = inputs["u"].shape[-1]
        parts = [{k: (v[..., a:a + piece] if k in seq else v[a:a + piece] if k in ("A", "D") else v)
                  for k, v in inputs.items()} for a in range(0, n, piece)]
        cat = {"y": -1, "du": -1, "ddelta": -1, "dz": -1, "dA": 0, "dD": 0}
        summed = ("dB", "dC")
    else:
        n = inputs["u"].shape[0]
        parts = [{k: (v[a:a + piece] if k in seq + ("B", "C") else v) for k, v in inputs.items()}
                 for a in range(0, n, piece)]
        cat = {"y": 0, "du": 0, "ddelta": 0, "dz": 0, "dB": 0, "dC": 0}
        summed = ("dA", "dD")
    ys, gs = [], []
    for p in parts:
        y, g = scan_ref.scan_vjp(p, gated=True, dtype=dtype)
        ys.append(y)
        gs.append(g)
    y = torch.cat(ys, dim=cat["y"])
    g = {k: torch.cat([x[k] for x in gs], dim=cat[k]) for k in cat if k != "y"}
    for k in summed:
        g[k] = torch.stack([x[k] for x in gs]).sum(0)
    return y, g
