"""The training caller on the device (python/diffrast/data.py:77-126,
python/train.py:127-179): synthetic scenes drawn as the reference draws them and
rendered in one launch per batch, and train_step's fused loss on CUDA tensors.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

from conftest import assert_images_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def test_synthetic_batches_render_the_reference_draws(oracle):
    from diffrast.data import DeviceBatches, SyntheticShapeDataset
    from diffrast.torch_layer import random_params

    ds = SyntheticShapeDataset(length=20, size=40, triangles=12, sigma=0.004, seed=3)
    # The draws: item i's generator, random_params then the background (data.py:111-115).
    gen = torch.Generator().manual_seed(3 * 1_000_003 + 7)
    p_ref = random_params(1, 12, generator=gen)
    bg_ref = torch.rand(3, generator=gen) * 0.3
    p, bg = ds.scene(7)
    assert torch.equal(p, p_ref) and torch.equal(bg, bg_ref)
    # One launch for a batch, per-scene backgrounds; equal to items one by one
    # and to the oracle's render of the same draws.
    batch = ds.batch([7, 2, 19])
    assert batch.is_cuda and batch.shape == (3, 3, 40, 40)
    assert torch.equal(batch[0], ds[7]) and torch.equal(batch[2], ds[19])
    ref = oracle.render_batch(p.numpy(), 40, 40, 0.004, bg.numpy())
    assert_images_close(batch[0].permute(1, 2, 0).cpu().numpy()[None], ref, "dataset item")
    seen = torch.cat(list(DeviceBatches(ds, 8)))
    assert seen.shape == (20, 3, 40, 40) and torch.equal(seen[7], ds[7])
    halves = [torch.cat(list(DeviceBatches(ds, 8, rank=r, world_size=2))) for r in range(2)]
    assert halves[0].shape[0] + halves[1].shape[0] == 20
    assert torch.equal(halves[1][0], ds[1])


def test_train_step_on_device_tensors_descends():
    from diffrast import train
    from diffrast.data import SyntheticShapeDataset
    from diffrast.torch_layer import activate, fused_mse, rasterize

    dev = torch.device("cuda", 0)
    ds = SyntheticShapeDataset(length=16, size=32, triangles=8, sigma=0.004, seed=1)
    images = ds.batch(range(16))
    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Flatten(), torch.nn.Linear(3 * 32 * 32, 8 * 10)).to(dev)

    class Model(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.net = net

        def forward(self, x):
            return activate(self.net(x).reshape(-1, 8, 10))

    model = Model()
    # fused_mse equals F.mse_loss(rasterize(...)) on device tensors (the
    # reference's test_fused_mse_matches_rasterize_then_mse).
    with torch.no_grad():
        pred = model(images)
    a = fused_mse(pred, images, sigma=0.004)
    b = torch.nn.functional.mse_loss(rasterize(pred, 32, 32, 0.004), images)
    torch.testing.assert_close(a, b, rtol=1e-5, atol=0)

    opt = torch.optim.Adam(model.parameters(), lr=3e-3)
    args = SimpleNamespace(param_weight=0.0, render_weight=1.0, render_fraction=1.0,
                           raster_device="auto")
    losses = []
    for _ in range(25):
        opt.zero_grad()
        loss, metrics = train.train_step(model, images, args, 0.004, dev)
        loss.backward()
        opt.step()
        losses.append(metrics["render_loss"])
        assert loss.is_cuda and np.isfinite(metrics["psnr"])
    assert losses[-1] < 0.8 * losses[0]


def test_global_fused_mse_matches_the_full_batch_on_one_gpu():
    # Two "ranks" on one GPU: each half's gradient under global_fused_mse
    # equals the full-batch mean's gradient on that half.
    from diffrast import train
    from diffrast.scenes import uniform_scenes
    from diffrast.torch_layer import fused_mse

    p = torch.from_numpy(uniform_scenes(8, 30, 5)).cuda()
    tgt = torch.rand(8, 3, 24, 24, device="cuda")
    full = p.clone().requires_grad_(True)
    fused_mse(full, tgt).backward()
    parts = []
    for lo in (0, 4):
        q = p[lo:lo + 4].clone().requires_grad_(True)
        train.global_fused_mse(q, tgt[lo:lo + 4], global_batch=8).backward()
        parts.append(q.grad)
    torch.testing.assert_close(torch.cat(parts), full.grad, rtol=1e-5, atol=1e-10)
