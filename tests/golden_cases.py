"""Constructor arguments of the golden fixtures made by tests/golden/make_golden.py."""

import os

import torch

from conftest import GOLDEN

SCAN_CASES = ["scan_b2_l7_d8", "scan_b1_l33_d12_randA", "scan_b2_l40_d40_plain", "scan_b1_l1_d4"]

# name -> (kind, kwargs)
MODULE_CASES = {
    "mamba_block_d16_l10": ("mamba", dict(d_model=16, d_state=16, d_conv=4, expand_factor=2)),
    "bidir_d8_l9": ("bidir", dict(d_model=8, d_state=16, d_conv=4, expand_factor=2)),
    "multidir_k2": ("multidir", dict(d_model=8, num_directions=2, grid_shape=(12,))),
    "multidir_k4": ("multidir", dict(d_model=8, num_directions=4, grid_shape=(3, 4))),
    "multidir_k6": ("multidir", dict(d_model=8, num_directions=6, grid_shape=(2, 3, 2))),
    "multidir_k8": ("multidir", dict(d_model=8, num_directions=8, grid_shape=(2, 2, 3, 2))),
    "multidir_k4_subset": ("multidir", dict(d_model=8, num_directions=4, grid_shape=(3, 4))),
    "vision_mamba_2d": ("vision", dict(img_size=8, patch_size=4, in_channels=1, embed_dim=8, depth=1, input_dim=2)),
    "vision_mamba_3d": ("vision", dict(img_size=8, patch_size=4, in_channels=1, embed_dim=8, depth=1, input_dim=3)),
    "vision_mamba_4d": (
        "vision",
        dict(img_size=8, patch_size=4, in_channels=1, embed_dim=8, depth=1, input_dim=4, num_temporal_frames=2),
    ),
}


def load(name):
    return torch.load(os.path.join(GOLDEN, name + ".pt"))


def build(kind, kwargs, lib):
    """Instantiate the fixture's module from `lib` (the oracle or the product)."""
    if lib == "oracle":
        from oracle import model_ref as m

        table = {
            "mamba": m.MambaBlockRef,
            "bidir": m.BidirectionalMambaBlockRef,
            "multidir": m.MultiDirectionalMambaBlockRef,
            "vision": m.VisionMambaRef,
        }
    else:
        import mlx_vision_mamba_b200 as m

        table = {
            "mamba": m.MambaBlock,
            "bidir": m.BidirectionalMambaBlock,
            "multidir": m.MultiDirectionalMambaBlock,
            "vision": m.VisionMamba,
        }
    return table[kind](**kwargs)


def load_params(module, params):
    sd = module.state_dict()
    missing = set(sd) - set(params)
    extra = set(params) - set(sd)
    assert not missing and not extra, (missing, extra)
    module.load_state_dict({k: v.reshape(sd[k].shape) for k, v in params.items()})
