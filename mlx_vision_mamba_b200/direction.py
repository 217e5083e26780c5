"""Scan directions of the multi-directional Mamba blocks, as index descriptors.

The reference builds, for each direction, a permuted (and possibly flipped)
copy of the sequence, runs the block on it and undoes the permutation
(mlx_vision_mamba/mamba_block.py:244-338 helpers, :407-534 `_apply_direction`).
Here a direction is only a descriptor: the token grid, the axis order of the
scan and a reverse flag.  The CUDA kernels map scan position -> token on the
fly (TMA tensor maps for the scan, integer maths for the conv), so no permuted
copy is ever made.

Semantics: tokens are laid out row-major on ``grid``; the scan visits them in
the order of ``transpose(grid, axes)`` flattened row-major, reversed when
``reverse`` is set.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

from . import _native


@dataclass(frozen=True)
class ScanDirection:
    grid: Tuple[int, ...] = ()
    axes: Tuple[int, ...] = ()
    reverse: bool = False

    def __post_init__(self):
        if len(self.grid) != len(self.axes):
            raise ValueError(f"grid {self.grid} and axes {self.axes} must have the same length")
        if len(self.grid) > 4:
            raise ValueError("at most 4 grid dims are supported")
        if sorted(self.axes) != list(range(len(self.axes))):
            raise ValueError(f"axes {self.axes} is not a permutation")

    @property
    def is_identity(self) -> bool:
        return not self.reverse and tuple(self.axes) == tuple(sorted(self.axes))

    def to_native(self) -> "_native.Direction":
        return _native.make_direction(len(self.grid), self.grid, self.axes, self.reverse)

    def scan_order(self, seqlen: int) -> List[int]:
        """Token index visited at each scan step (host-side helper for tests and tools)."""
        if not self.grid:
            order = list(range(seqlen))
        else:
            n = 1
            for g in self.grid:
                n *= g
            if n != seqlen:
                raise ValueError(f"grid {self.grid} does not cover {seqlen} tokens")
            strides = [1] * len(self.grid)
            for i in range(len(self.grid) - 2, -1, -1):
                strides[i] = strides[i + 1] * self.grid[i + 1]
            pshape = [self.grid[a] for a in self.axes]
            order = []
            idx = [0] * len(pshape)
            for _ in range(seqlen):
                order.append(sum(idx[q] * strides[self.axes[q]] for q in range(len(pshape))))
                for q in range(len(pshape) - 1, -1, -1):
                    idx[q] += 1
                    if idx[q] < pshape[q]:
                        break
                    idx[q] = 0
        return order[::-1] if self.reverse else order


FORWARD = ScanDirection()
BACKWARD = ScanDirection(reverse=True)

# Axis orders of the reference (mamba_block.py:478-482 for K=6, :508-513 for K=8).
_AXIS_PERMS = {
    4: [(0, 1), (1, 0)],
    6: [(0, 1, 2), (1, 0, 2), (2, 0, 1)],
    8: [(0, 1, 2, 3), (1, 0, 2, 3), (2, 0, 1, 3), (3, 0, 1, 2)],
}


def directions_for(num_directions: int, grid_shape: Optional[Sequence[int]] = None) -> List[ScanDirection]:
    """The K directions of MultiDirectionalMambaBlock, in the reference's block order.

    Direction 2p is axis order p forward and 2p+1 the same order reversed
    (mamba_block.py:450-534).  K=2 is forward + backward on the flat sequence.
    """
    if num_directions == 2:
        return [FORWARD, BACKWARD]
    if num_directions not in _AXIS_PERMS:
        raise ValueError(f"num_directions must be 2, 4, 6, or 8, got {num_directions}")
    grid = tuple(int(g) for g in grid_shape)
    out = []
    for perm in _AXIS_PERMS[num_directions]:
        if len(perm) != len(grid):
            raise ValueError(f"K={num_directions} requires a {len(perm)}-D grid, got {grid}")
        for rev in (False, True):
            out.append(ScanDirection(grid=grid, axes=tuple(perm), reverse=rev))
    return out
