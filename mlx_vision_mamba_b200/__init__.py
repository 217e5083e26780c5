"""B200-native (sm_100a) selective-scan hot path of mlx-vision-mamba.

Same public names as `mlx_vision_mamba` (its __init__.py:7-33), backed by
hand-written CUDA kernels in libvmscan.so (C ABI: include/vmscan.h) for the
selective scan, its VJP, the SiLU gate and the direction-aware causal conv1d.
"""

from .direction import BACKWARD, FORWARD, ScanDirection, directions_for
from .mamba_block import (
    BidirectionalMambaBlock,
    MambaBlock,
    MultiDirectionalMambaBlock,
    ResidualMambaBlock,
)
from .scan import (
    conv1d_silu_cuda,
    device_status,
    dt_softplus_cuda,
    selective_scan,
    selective_scan_cuda,
    selective_scan_metal,
    selective_scan_metal_fused,
    selective_scan_metal_trainable,
)
from .vision_mamba import PatchEmbed, PatchEmbed3D, PatchEmbed4D, VisionMamba

__version__ = "0.1.0"
__all__ = [
    "MambaBlock",
    "ResidualMambaBlock",
    "BidirectionalMambaBlock",
    "MultiDirectionalMambaBlock",
    "VisionMamba",
    "PatchEmbed",
    "PatchEmbed3D",
    "PatchEmbed4D",
    "ScanDirection",
    "FORWARD",
    "BACKWARD",
    "directions_for",
    "selective_scan",
    "dt_softplus_cuda",
    "selective_scan_cuda",
    "selective_scan_metal",
    "selective_scan_metal_trainable",
    "selective_scan_metal_fused",
    "conv1d_silu_cuda",
    "device_status",
]
