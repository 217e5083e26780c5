"""Data-parallel training step for the VisionMamba encoders.

The reference has no training loop or distributed code (it runs one MLX
device); this is the harness of the VisionMamba 2D / 3D / 4D training
configurations: a VisionMamba forward, an MSE loss against a target of the feature shape, backward and an
AdamW update, with the global batch split across one process per GPU and the
gradients averaged by DistributedDataParallel (bucketed NCCL all-reduce over
NVLink, overlapped with the backward).  Every function here is model-agnostic
so the data-parallel logic can be exercised on CPU ranks (gloo).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F


@dataclass(frozen=True)
class EncoderConfig:
    """A VisionMamba training configuration (2D K=4, 3D K=6 or 4D K=8 benchmark step)."""

    name: str
    input_shape: Tuple[int, ...]  # per-sample input, channel-last
    img_size: int
    patch_size: int
    embed_dim: int = 384
    depth: int = 6
    d_state: int = 16
    input_dim: int = 2
    num_temporal_frames: int = 1
    temporal_patch_size: int = 1
    global_batch: int = 64

    @property
    def num_tokens(self) -> int:
        g = self.img_size // self.patch_size
        if self.input_dim == 4:
            return (self.num_temporal_frames // self.temporal_patch_size) * g ** 3
        return g ** self.input_dim


VISION_MAMBA_2D = EncoderConfig("VisionMamba-2D K=4", (224, 224, 1), 224, 16, input_dim=2, global_batch=64)
VISION_MAMBA_3D = EncoderConfig("VisionMamba-3D K=6", (128, 128, 128, 1), 128, 16, input_dim=3, global_batch=16)
VISION_MAMBA_4D = EncoderConfig(
    "VisionMamba-4D K=8", (8, 64, 64, 64, 1), 64, 16, input_dim=4, num_temporal_frames=8, global_batch=8
)


def shard(global_batch: int, rank: int, world: int) -> Tuple[int, int]:
    """[start, stop) of this rank's slice of the global batch (contiguous, balanced)."""
    if global_batch < world:
        raise ValueError(f"global batch {global_batch} smaller than world size {world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def synthetic_batch(cfg: EncoderConfig, batch: int, device, seed: int):
    """Seeded N(0,1) inputs and MSE targets of the config's shapes."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((batch, *cfg.input_shape), generator=g, device=device)
    target = torch.randn((batch, cfg.num_tokens, cfg.embed_dim), generator=g, device=device)
    return x, target


def build_encoder(cfg: EncoderConfig, device, seed: int = 0):
    from .vision_mamba import VisionMamba

    torch.manual_seed(seed)
    return VisionMamba(
        img_size=cfg.img_size, patch_size=cfg.patch_size, in_channels=cfg.input_shape[-1],
        embed_dim=cfg.embed_dim, depth=cfg.depth, d_state=cfg.d_state, input_dim=cfg.input_dim,
        num_temporal_frames=cfg.num_temporal_frames, temporal_patch_size=cfg.temporal_patch_size,
    ).to(device)


def wrap_data_parallel(model: torch.nn.Module, device: Optional[torch.device] = None):
    """DDP when a process group with more than one rank is active, else the model itself.

    The gradients are views into DDP's all-reduce buckets (no copy into and out
    of the buckets around each all-reduce): on 2 GPUs the VisionMamba-2D step
    took 12.03 ms against 12.52 ms with copied buckets (25 MB buckets; 10 and
    100 MB buckets measured no better)."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        ids = [device.index] if device is not None and device.type == "cuda" else None
        return torch.nn.parallel.DistributedDataParallel(model, device_ids=ids, bucket_cap_mb=25,
                                                         gradient_as_bucket_view=True)
    return model


def train_step(model, optimizer, x, target) -> torch.Tensor:
    """One step: forward, MSE against the target, backward (gradients averaged
    across ranks by DDP), AdamW update.  Returns the detached loss."""
    out = model(x)
    loss = F.mse_loss(out, target)
    optimizer.zero_grad(set_to_none=True)
    loss.backward()
    optimizer.step()
    return loss.detach()


def _unwrap(model: torch.nn.Module) -> torch.nn.Module:
    return model.module if isinstance(model, torch.nn.parallel.DistributedDataParallel) else model


def save_checkpoint(path: str, model: torch.nn.Module, optimizer=None, step: int = 0) -> None:
    """torch.save of the model's state dict (unwrapped from DDP, so a checkpoint
    loads into a single-GPU model too), the optimizer's state and the step.
    Under a process group only rank 0 writes; all ranks hold the same
    parameters after DDP's all-reduce."""
    if dist.is_available() and dist.is_initialized() and dist.get_rank() != 0:
        return
    torch.save({"model": _unwrap(model).state_dict(),
                "optimizer": optimizer.state_dict() if optimizer is not None else None,
                "step": int(step)}, path)


def load_checkpoint(path: str, model: torch.nn.Module, optimizer=None, map_location=None) -> int:
    """Restores what save_checkpoint wrote (every rank reads the file) and
    returns the saved step."""
    ck = torch.load(path, map_location=map_location, weights_only=True)
    _unwrap(model).load_state_dict(ck["model"])
    if optimizer is not None and ck.get("optimizer") is not None:
        optimizer.load_state_dict(ck["optimizer"])
    return int(ck.get("step", 0))


def make_optimizer(model, lr: float = 1e-4, capturable: bool = False):
    """AdamW; `capturable` keeps its step counters on the device so the
    update can be replayed inside a CUDA graph.  Parameters on the GPU use
    PyTorch's fused AdamW (one pass over parameters, gradients and moments
    instead of the multi-tensor implementation's several)."""
    params = list(model.parameters())
    fused = bool(params) and all(p.is_cuda for p in params)
    return torch.optim.AdamW(params, lr=lr, weight_decay=0.05, capturable=capturable, fused=fused)


def check_device_status(device=None) -> None:
    """Raise if a kernel of libvmscan.so gave up a bounded device-side wait
    since the last check (VMSCAN_ERR_TIMEOUT): its outputs are then wrong.
    Synchronises the device's current stream; clears the status."""
    from . import _native
    from .scan import device_status

    st = device_status(device, clear=True)
    if st != 0:
        raise _native.VmscanError(st, "device status after training steps")


class GraphedTrainStep:
    """The whole training step (forward, MSE, backward with DDP's gradient
    all-reduce, AdamW update) captured once into a CUDA graph and replayed:
    one graph launch per step instead of hundreds of kernel launches and the
    Python autograd work around them, so small per-GPU batches stay GPU-bound.

    Inputs are copied into static buffers before each replay.  The model must
    be wrapped by `wrap_data_parallel` inside `side_stream` (DDP's documented
    requirement for capture) and the optimizer built with `capturable=True`.
    `warmup` eager steps run on the side stream first (DDP needs at least 11
    before its buckets are final); the parameters, buffers and optimizer state
    are restored afterwards, so the first replay is the model's first update.
    Every `status_every` replays (and in `close()`) the device status of the
    scan kernels is checked, which raises on a timed-out device wait.
    Release the step (`close()`) before destroying a process group whose
    collectives it captured.
    """

    def __init__(self, model, optimizer, x, target, side_stream=None, warmup: int = 11, status_every: int = 100):
        self.model, self.optimizer = model, optimizer
        self.device = x.device
        self.status_every = int(status_every)
        self.replays = 0
        self.x = x.detach().clone()
        self.target = target.detach().clone()
        saved = _snapshot(model, optimizer)
        stream = side_stream if side_stream is not None else torch.cuda.Stream(device=x.device)
        stream.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                train_step(model, optimizer, self.x, self.target)
            # the warm-up steps only settle DDP's buckets and create the
            # optimizer state; undo their updates in place (the graph
            # captures these tensors' addresses)
            _restore(model, optimizer, saved)
        torch.cuda.current_stream(x.device).wait_stream(stream)
        optimizer.zero_grad(set_to_none=True)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            out = model(self.x)
            self.loss = F.mse_loss(out, self.target)
            self.loss.backward()
            optimizer.step()

    def __call__(self, x=None, target=None) -> torch.Tensor:
        if x is not None:
            self.x.copy_(x, non_blocking=True)
        if target is not None:
            self.target.copy_(target, non_blocking=True)
        self.graph.replay()
        self.replays += 1
        if self.status_every > 0 and self.replays % self.status_every == 0:
            check_device_status(self.device)
        return self.loss

    def close(self) -> None:
        if self.graph is not None:
            check_device_status(self.device)
        self.graph = None


def _snapshot(model, optimizer):
    """Copies of the parameters, buffers and optimizer state (tensors cloned)."""
    with torch.no_grad():
        params = [p.detach().clone() for p in model.parameters()]
        bufs = [b.detach().clone() for b in model.buffers()]
        state = {p: {k: (v.detach().clone() if torch.is_tensor(v) else v) for k, v in st.items()}
                 for p, st in optimizer.state.items()}
    return params, bufs, state


def _restore(model, optimizer, saved) -> None:
    """Puts back what `_snapshot` saved, in place.  Optimizer state created
    after the snapshot (a fresh optimizer's first steps) is reset to zero,
    the value a fresh AdamW starts from."""
    params, bufs, state = saved
    with torch.no_grad():
        for p, v in zip(model.parameters(), params):
            p.copy_(v)
        for b, v in zip(model.buffers(), bufs):
            b.copy_(v)
        for p, st in optimizer.state.items():
            old = state.get(p, {})
            for k, v in st.items():
                if torch.is_tensor(v):
                    if k in old:
                        v.copy_(old[k])
                    else:
                        v.zero_()
                elif k in old:
                    st[k] = old[k]
