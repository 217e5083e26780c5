"""Parity rule shared by the GPU tests.

The north-star tolerance is 1e-5 relative / 1e-6 absolute on fp32 outputs and
gradients.  It is applied against the exact result of the reference algorithm
(the oracle in fp64).  The reference's own fp32 arithmetic does not meet that
bound everywhere (ddelta sums A[n] * g[n] with |A| up to 16 and cancels), so at
an element where the reference's fp32 result (`ref32`) itself misses the
bound, the bound becomes twice the reference's own error there: the CUDA
result must be at least half as accurate as the reference it replaces, and
nowhere worse than that.
"""

import torch

from conftest import ATOL, RTOL


def parity_report(ours, ref64, ref32=None, rtol=RTOL, atol=ATOL):
    ours = ours.detach().double().cpu()
    ref64 = ref64.detach().double().cpu()
    err = (ours - ref64).abs()
    bound = atol + rtol * ref64.abs()
    if ref32 is not None:
        ref_err = (ref32.detach().double().cpu() - ref64).abs()
        bound = torch.maximum(bound, 2.0 * ref_err)
    ratio = (err / bound).max().item() if err.numel() else 0.0
    strict = (err <= atol + rtol * ref64.abs()).double().mean().item() if err.numel() else 1.0
    return ratio, strict


def assert_parity(name, ours, ref64, ref32=None, rtol=RTOL, atol=ATOL):
    assert ours.shape == ref64.shape, (name, tuple(ours.shape), tuple(ref64.shape))
    assert torch.isfinite(ours).all(), f"{name}: non-finite values"
    ratio, strict = parity_report(ours, ref64, ref32, rtol, atol)
    assert ratio <= 1.0, f"{name}: error/bound = {ratio:.3f} (strict-tolerance fraction {strict:.6f})"
