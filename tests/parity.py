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


def parity_report(ours, ref64, ref32=None, rtol=RTOL, atol=ATOL):
    ours = ours.detach().double().cpu()
    ref64 = ref64.detach().double().cpu()
    err = (ours - ref64).abs()
    strict_bound = atol + rtol * ref64.abs()
    bound = strict_bound
    norm_ok = True
    norm_ratio = 0.0
    if ref32 is not None:
        ref_err = (ref32.detach().double().cpu() - ref64).abs()
        bound = strict_bound + 2.0 * (ref_err.max() if ref_err.numel() else 0.0)
        lhs = err.norm().item()
        rhs = 2.0 * ref_err.norm().item() + atol * math.sqrt(max(err.numel(), 1))
        norm_ratio = lhs / rhs
        norm_ok = lhs <= rhs
    ratio = (err / bound).max().item() if err.numel() else 0.0
    strict = (err <= strict_bound).double().mean().item() if err.numel() else 1.0
    return ratio, strict, norm_ok, norm_ratio


def assert_parity(name, ours, ref64, ref32=None, rtol=RTOL, atol=ATOL):
    assert ours.shape == ref64.shape, (name, tuple(ours.shape), tuple(ref64.shape))
    assert torch.isfinite(ours).all(), f"{name}: non-finite values"
    ratio, strict, norm_ok, norm_ratio = parity_report(ours, ref64, ref32, rtol, atol)
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
