"""Checkpoint / resume of the training harness (torch.save of the state
dicts): a CPU round trip of the model and optimizer, and on the GPU a resumed
run that continues exactly where the saved one stopped."""

import pytest
import torch

from mlx_vision_mamba_b200 import train


def small_cfg():
    return train.EncoderConfig("tiny 2D", (64, 64, 1), 64, 16, embed_dim=32, depth=2, input_dim=2, global_batch=2)


def test_checkpoint_round_trip_cpu(tmp_path):
    cfg = small_cfg()
    m = train.build_encoder(cfg, "cpu", seed=0)
    opt = train.make_optimizer(m, lr=3e-4)
    path = str(tmp_path / "ck.pt")
    train.save_checkpoint(path, m, opt, step=7)
    ref = {k: v.clone() for k, v in m.state_dict().items()}
    with torch.no_grad():
        for p in m.parameters():
            p.add_(1.0)
    m2 = train.build_encoder(cfg, "cpu", seed=5)
    opt2 = train.make_optimizer(m2, lr=1e-1)
    assert train.load_checkpoint(path, m2, opt2) == 7
    for k, v in m2.state_dict().items():
        assert torch.equal(v, ref[k]), k
    assert opt2.param_groups[0]["lr"] == 3e-4


@pytest.mark.gpu
def test_resume_continues_the_run(tmp_path):
    cfg = small_cfg()
    dev = torch.device("cuda", 0)
    x, tgt = train.synthetic_batch(cfg, 2, dev, seed=1)
    m = train.build_encoder(cfg, dev, seed=0)
    opt = train.make_optimizer(m)
    for _ in range(2):
        train.train_step(m, opt, x, tgt)
    path = str(tmp_path / "ck.pt")
    train.save_checkpoint(path, m, opt, step=2)
    losses = [train.train_step(m, opt, x, tgt).item() for _ in range(2)]
    m2 = train.build_encoder(cfg, dev, seed=3)
    opt2 = train.make_optimizer(m2)
    assert train.load_checkpoint(path, m2, opt2, map_location=dev) == 2
    resumed = [train.train_step(m2, opt2, x, tgt).item() for _ in range(2)]
    assert resumed == losses


def test_warmup_snapshot_restores_model_and_optimizer_cpu():
    """GraphedTrainStep's warm-up undo (train._snapshot / _restore) on CPU: after
    steps that create the optimizer state, the parameters are back to their
    values and the fresh state reads as a new AdamW's (zero moments and step),
    so the next update equals a fresh optimizer's first update."""
    lin = torch.nn.Linear(8, 4)
    opt = torch.optim.AdamW(lin.parameters(), lr=1e-2)
    ref = torch.nn.Linear(8, 4)
    ref.load_state_dict(lin.state_dict())
    ref_opt = torch.optim.AdamW(ref.parameters(), lr=1e-2)
    x = torch.randn(5, 8)
    saved = train._snapshot(lin, opt)
    for _ in range(3):
        opt.zero_grad()
        lin(x).square().sum().backward()
        opt.step()
    assert not torch.equal(lin.weight, ref.weight)
    train._restore(lin, opt, saved)
    assert torch.equal(lin.weight, ref.weight) and torch.equal(lin.bias, ref.bias)
    for st in opt.state.values():
        assert all(float(v.abs().sum()) == 0.0 for v in st.values() if torch.is_tensor(v))
    for m, o in ((lin, opt), (ref, ref_opt)):
        o.zero_grad()
        m(x).square().sum().backward()
        o.step()
    assert torch.equal(lin.weight, ref.weight) and torch.equal(lin.bias, ref.bias)
