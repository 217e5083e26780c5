"""Data-parallel logic on CPU ranks (gloo, world size 2): sharding, gradient
averaging and the max-over-ranks timing reduction used by bench.py.  The model
is the CPU oracle (the product model has no CPU path); the DP code under test
is model-agnostic."""

import os
import socket

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
