"""Data-parallel logic on CPU ranks (gloo, world size 2): sharding, gradient
averaging and the max-over-ranks timing reduction used by bench.py.  The model
is the CPU oracle (the product model has no CPU path); the DP code under test
is model-agnostic."""

import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mlx_vision_mamba_b200 import train


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_covers_batch_once():
    for gb in (8, 9, 64):
        for world in (1, 2, 3, 8):
            if gb < world:
                continue
            spans = [train.shard(gb, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == gb
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        train.shard(2, 0, 4)


def _tiny_model():
    from oracle.model_ref import VisionMambaRef

    torch.manual_seed(0)
    return VisionMambaRef(img_size=8, patch_size=4, in_channels=1, embed_dim=8, depth=1, input_dim=2)


def _worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = train.wrap_data_parallel(_tiny_model())
        g = torch.Generator().manual_seed(123)
        x = torch.randn(4, 8, 8, 1, generator=g)
        tgt = torch.randn(4, 4, 8, generator=g)
        a, b = train.shard(4, rank, world)
        out = model(x[a:b])
        loss = torch.nn.functional.mse_loss(out, tgt[a:b])
        loss.backward()
        grads = {k: p.grad.clone() for k, p in model.module.named_parameters()}
        t = torch.tensor([float(rank + 1)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            torch.save({"grads": grads, "tmax": t.item()}, out_path)
    finally:
        dist.destroy_process_group()


def test_ddp_gradients_equal_full_batch(tmp_path):
    world = 2
    out_path = str(tmp_path / "g.pt")
    mp.spawn(_worker, args=(world, _free_port(), out_path), nprocs=world, join=True)
    rec = torch.load(out_path)
    assert rec["tmax"] == 2.0
    model = _tiny_model()
    g = torch.Generator().manual_seed(123)
    x = torch.randn(4, 8, 8, 1, generator=g)
    tgt = torch.randn(4, 4, 8, generator=g)
    torch.nn.functional.mse_loss(model(x), tgt).backward()
    for k, p in model.named_parameters():
        torch.testing.assert_close(rec["grads"][k], p.grad, rtol=1e-5, atol=1e-6)


class _FakeBranchBlock(torch.nn.Module):
    """Stands in for a MambaBlock on the CPU (the scan kernels are CUDA-only):
    the same projection parameters and `scan_branch` interface, with an
    elementwise, direction-dependent body."""

    def __init__(self, d_model, d_inner, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.d_inner = d_inner
        self.in_proj = torch.nn.Linear(d_model, 2 * d_inner, bias=False)
        self.out_proj = torch.nn.Linear(d_inner, d_model, bias=False)
        with torch.no_grad():
            self.in_proj.weight.copy_(torch.randn(2 * d_inner, d_model, generator=g) * 0.3)
            self.out_proj.weight.copy_(torch.randn(d_model, d_inner, generator=g) * 0.3)

    def scan_branch(self, xz, direction):
        x, z = torch.split(xz, [self.d_inner, self.d_inner], dim=-1)
        y = torch.cumsum(torch.tanh(x), dim=1) if direction is None else torch.tanh(x).flip(1).cumsum(1).flip(1)
        return y * torch.sigmoid(z)

    def forward(self, h, direction=None):
        return self.out_proj(self.scan_branch(self.in_proj(h), direction))


def _directional_block(k):
    from mlx_vision_mamba_b200.direction import BACKWARD
    from mlx_vision_mamba_b200.mamba_block import MultiDirectionalMambaBlock

    torch.manual_seed(0)
    blk = MultiDirectionalMambaBlock(8, 16, 4, 2, num_directions=k, grid_shape=(4, 4) if k == 4 else None)
    blk.mamba_blocks = torch.nn.ModuleList([_FakeBranchBlock(8, 16, seed=10 + i) for i in range(k)])
    blk.directions = [None if i % 2 == 0 else BACKWARD for i in range(k)]
    return blk


def _shard_worker(rank, world, port, out_path, k):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        blk = _directional_block(k)
        blk.shard_directions(dist.group.WORLD)
        g = torch.Generator().manual_seed(7)
        x = torch.randn(2, 16, 8, generator=g).requires_grad_(True)
        dy = torch.randn(2, 16, 8, generator=g)
        y = blk(x)
        (y * dy).sum().backward()
        grads = {n: (p.grad.clone() if p.grad is not None else None) for n, p in blk.named_parameters()}
        torch.save({"y": y.detach(), "dx": x.grad.clone(), "grads": grads}, f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("k", [2, 4])
def test_direction_sharding_matches_unsharded(tmp_path, k):
    """Directions split over 2 gloo ranks, summed by an autograd all-reduce:
    every rank gets the unsharded output and input gradient; each direction's
    parameters get their unsharded gradient on the rank that owns them; the
    shared LayerNorm's gradient is the same on every rank."""
    world = 2
    out_path = str(tmp_path / "shard")
    mp.spawn(_shard_worker, args=(world, _free_port(), out_path, k), nprocs=world, join=True)
    blk = _directional_block(k)
    g = torch.Generator().manual_seed(7)
    x = torch.randn(2, 16, 8, generator=g).requires_grad_(True)
    dy = torch.randn(2, 16, 8, generator=g)
    y = blk(x)
    (y * dy).sum().backward()
    for r in range(world):
        rec = torch.load(f"{out_path}.{r}")
        torch.testing.assert_close(rec["y"], y.detach(), rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(rec["dx"], x.grad, rtol=1e-5, atol=1e-6)
        for n, p in blk.named_parameters():
            owner = n.startswith("mamba_blocks.") and int(n.split(".")[1]) % world == r
            shared = not n.startswith("mamba_blocks.")
            if owner or shared:
                torch.testing.assert_close(rec["grads"][n], p.grad, rtol=1e-5, atol=1e-6, msg=n)
            else:
                assert rec["grads"][n] is None, n


def _failing_rank_worker(rank, world, port, out_path):
    """Rank 1 dies between steps (before the gradient all-reduce of its next
    step); rank 0's next collective must end with an error within the process
    group's short timeout instead of waiting forever."""
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    model = train.wrap_data_parallel(_tiny_model())
    opt = torch.optim.SGD(model.parameters(), lr=0.1)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 8, 8, 1, generator=g)
    tgt = torch.randn(2, 4, 8, generator=g)
    train.train_step(model, opt, x, tgt)  # one healthy step on both ranks
    if rank == 1:
        os._exit(0)  # the rank leaves between steps, with nothing in flight
    t0 = time.monotonic()
    try:
        train.train_step(model, opt, x, tgt)
        outcome = "completed"
    except Exception as e:  # noqa: BLE001 - any backend error is the expected signal
        outcome = f"raised {type(e).__name__}"
    with open(out_path, "w") as f:
        f.write(f"{outcome} {time.monotonic() - t0:.1f}")
    os._exit(0)


def test_lost_rank_surfaces_as_an_error_not_a_hang(tmp_path):
    out_path = str(tmp_path / "outcome.txt")
    mp.spawn(_failing_rank_worker, args=(2, _free_port(), out_path), nprocs=2, join=True)
    outcome, seconds = open(out_path).read().rsplit(" ", 1)
    assert outcome.startswith("raised"), outcome
    assert float(seconds) < 60.0
