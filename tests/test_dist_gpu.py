"""Direction parallelism of the VisionMamba encoder on 2 GPUs (NCCL): each rank
runs half of every layer's scan directions; outputs and gradients equal the
unsharded model's.  Skipped on boxes with fewer than 2 GPUs."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model(dev):
    from mlx_vision_mamba_b200 import VisionMamba

    torch.manual_seed(0)
    return VisionMamba(img_size=32, patch_size=8, in_channels=1, embed_dim=32, depth=2, input_dim=2).to(dev)


def _run(model, dev):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 32, 32, 1, generator=g).to(dev)
    dy = torch.randn(2, 16, 32, generator=g).to(dev)
    y = model(x)
    (y * dy).sum().backward()
    torch.cuda.synchronize(dev)
    return y.detach().cpu(), {n: (p.grad.detach().cpu() if p.grad is not None else None)
                              for n, p in model.named_parameters()}


def _worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        model = _model(dev)
        model.shard_directions(dist.group.WORLD)
        y, grads = _run(model, dev)
        torch.save({"y": y, "grads": grads}, f"{out_path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_direction_sharded_encoder_matches_unsharded(tmp_path):
    torch.backends.cuda.matmul.allow_tf32 = False
    out_path = str(tmp_path / "dirshard")
    mp.spawn(_worker, args=(2, _free_port(), out_path), nprocs=2, join=True)
    y_ref, g_ref = _run(_model(torch.device("cuda", 0)), torch.device("cuda", 0))
    for r in range(2):
        rec = torch.load(f"{out_path}.{r}")
        torch.testing.assert_close(rec["y"], y_ref, rtol=1e-4, atol=1e-5)
        for n, gr in g_ref.items():
            got = rec["grads"][n]
            k = int(n.split(".")[3]) if ".mamba_blocks." in n else None
            if k is None or k % 2 == r:
                torch.testing.assert_close(got, gr, rtol=1e-4, atol=1e-5, msg=n)
            else:
                assert got is None, n
