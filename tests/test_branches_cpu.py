"""Host logic of the fused K-branch node that runs without a GPU: the split-K
weight-gradient product a^T b sums its chunks in a fixed order and equals the
plain product for every token count (divisible or not, short or long)."""

import pytest
import torch

from mlx_vision_mamba_b200.branches import _mm_tn


@pytest.mark.parametrize("k", [1, 7, 255, 256, 300, 512, 1568, 3136, 6272, 12544, 12545])
def test_split_k_product_matches_plain_product(k):
    g = torch.Generator().manual_seed(k)
    a = torch.randn(k, 56, generator=g, dtype=torch.float64)
    b = torch.randn(k, 24, generator=g, dtype=torch.float64)
    torch.testing.assert_close(_mm_tn(a, b), a.t() @ b, rtol=1e-12, atol=1e-10)


def test_split_k_is_deterministic():
    g = torch.Generator().manual_seed(0)
    a = torch.randn(12544, 24, generator=g)
    b = torch.randn(12544, 56, generator=g)
    assert torch.equal(_mm_tn(a, b), _mm_tn(a, b))
