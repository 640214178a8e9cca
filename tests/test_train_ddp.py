"""Data-parallel plumbing of the training caller on two gloo ranks (CPU).

The rasterizer itself needs a GPU; here a CPU stand-in with the same contract
(mean over the batch of a per-scene loss, differentiable in the parameters)
takes its place, so these tests check only the scaling and the DDP wiring:
- global_fused_mse: each rank's gradient on its own scenes equals the gradient
  of the single-process mean over all B_global scenes (python/train.py:127-179
  under DDP, the benchmark's config 3 sharded over ranks);
- train_step under DistributedDataParallel: the averaged model gradient equals
  the single-process gradient on the whole batch.
"""

from __future__ import annotations

import os
import socket
from types import SimpleNamespace

import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG, REPO


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def stand_in_mse(params, targets, sigma=0.0015, background=(0.0, 0.0, 0.0)):
    # Mean over scenes of a smooth per-scene loss of params and targets.
    per = ((params.flatten(1) ** 2).sum(1) * 1e-2 + targets.flatten(1).mean(1) *
           params.flatten(1).sum(1) * 1e-3)
    return per.mean()


def _batch():
    g = torch.Generator().manual_seed(0)
    return torch.rand(8, 5, 10, generator=g), torch.rand(8, 3, 6, 6, generator=g)


class TinyNet(torch.nn.Module):
    def __init__(self):
        super().__init__()
        torch.manual_seed(1)
        self.lin = torch.nn.Linear(3 * 6 * 6, 5 * 10)

    def forward(self, images):
        return torch.sigmoid(self.lin(images.flatten(1))).reshape(-1, 5, 10)


def _worker(rank, world, port, out):
    import sys

    for p in (REPO, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    from diffrast import train

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    train.fused_mse = stand_in_mse
    params, targets = _batch()
    lo, hi = rank * 4, (rank + 1) * 4
    p = params[lo:hi].clone().requires_grad_(True)
    loss = train.global_fused_mse(p, targets[lo:hi], global_batch=8)
    loss.backward()
    total = loss.detach().clone()
    dist.all_reduce(total)

    model = torch.nn.parallel.DistributedDataParallel(TinyNet())
    args = SimpleNamespace(param_weight=0.0, render_weight=1.0, render_fraction=1.0,
                           raster_device="auto")
    step_loss, metrics = train.train_step(model, targets[lo:hi], args, 0.004,
                                          torch.device("cpu"))
    step_loss.backward()
    out[rank] = (p.grad.tolist(), total.item(),
                 [q.grad.clone().reshape(-1).tolist() for q in model.parameters()],
                 metrics["render_loss"])
    dist.destroy_process_group()


def test_global_batch_scaling_and_ddp_train_step_on_two_ranks():
    import sys

    for p in (REPO, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    from diffrast import train

    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
        for pr in procs:
            pr.start()
        for pr in procs:
            pr.join(120)
            assert pr.exitcode == 0
        res = [out[0], out[1]]

    params, targets = _batch()
    # Single process, the whole batch of 8.
    p = params.clone().requires_grad_(True)
    full = stand_in_mse(p, targets)
    full.backward()
    g0 = torch.tensor(res[0][0])
    g1 = torch.tensor(res[1][0])
    torch.testing.assert_close(torch.cat([g0, g1]), p.grad, rtol=1e-6, atol=1e-9)
    assert abs(res[0][1] - full.item()) < 1e-6 and res[0][1] == res[1][1]

    orig = train.fused_mse
    train.fused_mse = stand_in_mse
    try:
        model = TinyNet()
        args = SimpleNamespace(param_weight=0.0, render_weight=1.0, render_fraction=1.0,
                               raster_device="auto")
        loss, _ = train.train_step(model, targets, args, 0.004, torch.device("cpu"))
        loss.backward()
    finally:
        train.fused_mse = orig
    for a, b, q in zip(res[0][2], res[1][2], model.parameters()):
        assert a == b  # DDP leaves every rank with the same averaged gradient
        torch.testing.assert_close(torch.tensor(a), q.grad.reshape(-1), rtol=1e-5, atol=1e-8)


def test_global_fused_mse_rejects_a_smaller_global_batch():
    import sys

    for p in (REPO, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    from diffrast import train

    with pytest.raises(ValueError):
        train.global_fused_mse(torch.zeros(4, 2, 10), torch.zeros(4, 3, 2, 2), global_batch=2)
