"""Row-sharded single-scene path (benchmark config 4).

CPU: the shard partition covers every tile row once, and the all-reduce
plumbing gives every rank the same summed gradient (gloo, world size 2, with
the native call replaced by a deterministic fake). GPU: the sum over shards of
dr_loss_backward_sharded equals dr_loss_backward on the full scene, and on a
box with two GPUs the NCCL version of the step matches one GPU.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG, REPO, assert_grads_close


def test_shard_rows_cover_every_tile_row_once():
    from diffrast.sharded import shard_rows

    for height in (1, 15, 16, 17, 256, 1024, 1000):
        tiles = (height + 15) // 16
        for n in (1, 2, 3, 4, 8):
            rows = sorted(r for s in range(n) for r in shard_rows(height, s, n))
            assert rows == list(range(tiles)), (height, n)
    with pytest.raises(ValueError):
        shard_rows(64, 2, 2)


def test_pack_unpack_round_trip():
    from diffrast.sharded import pack_for_reduce, unpack_reduced

    g = torch.randn(2, 7, 10)
    s = torch.tensor([1.5, 2.5], dtype=torch.float64)
    buf = pack_for_reduce(g, s)
    g2, s2 = unpack_reduced(buf, g.shape, 2)
    assert torch.equal(g2, g) and torch.equal(s2, s)


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _gloo_worker(rank, world, port, out):
    import sys

    for p in (REPO, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    from diffrast import _native, sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)

    def fake(params, targets, sigma, shard, n_shards, background=(0.0, 0.0, 0.0)):
        # Partial results depend on the shard, like the kernel's.
        g = torch.full(params.shape, float(shard + 1)) * torch.arange(params.numel()).reshape(
            params.shape)
        return torch.tensor([10.0 * (shard + 1)], dtype=torch.float64), g

    _native.loss_backward_sharded = fake
    step = sharded.ShardedSceneStep(torch.zeros(1, 3, 10))
    losses, grads = step.loss_and_grads(torch.zeros(1, 4, 4, 3), 0.01)
    out[rank] = (losses.tolist(), grads.reshape(-1).tolist())
    dist.destroy_process_group()


def test_allreduce_plumbing_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        l0, g0 = out[0]
        l1, g1 = out[1]
    assert l0 == l1 and g0 == g1
    expect = [3.0 * i for i in range(30)]  # shard weights 1 + 2
    assert g0 == expect
    assert abs(l0[0] - 30.0 / 48.0) < 1e-6  # (10 + 20) / (4*4*3)


@pytest.mark.gpu
@pytest.mark.parametrize("n_shards", [2, 4, 8])
def test_sum_over_shards_equals_the_full_scene(n_shards):
    from diffrast import _native
    from diffrast.scenes import config4_params

    p = torch.from_numpy(config4_params(4096, 4000)).cuda()
    tp = torch.from_numpy(config4_params(4096, 4001)).cuda()
    target = _native.render(tp, 1024, 1024, 0.0015)
    losses, grads = _native.loss_backward(p, target, 0.0015)
    total_g = torch.zeros_like(grads, dtype=torch.float64)
    total_s = torch.zeros(1, dtype=torch.float64, device="cuda")
    for s in range(n_shards):
        sums, g = _native.loss_backward_sharded(p, target, 0.0015, s, n_shards)
        total_g += g.double()
        total_s += sums
    mse = (total_s / (1024 * 1024 * 3)).float()
    torch.testing.assert_close(mse, losses, rtol=1e-6, atol=0)
    assert_grads_close(total_g.float().cpu().numpy(), grads.cpu().numpy(), "sharded sum")


def _nccl_worker(rank, world, port, out):
    import sys

    for p in (REPO, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist

    from diffrast import _native, sharded
    from diffrast.scenes import config4_params

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    p = torch.from_numpy(config4_params(1024, 4000)).cuda()
    target = _native.render(torch.from_numpy(config4_params(1024, 4001)).cuda(), 512, 512,
                            0.0015)
    step = sharded.ShardedSceneStep(p)
    for _ in range(3):
        losses = step.step(target, 0.0015)
    torch.cuda.synchronize()
    out[rank] = (losses.cpu().tolist(), step.params.cpu().numpy().tolist())
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_gpu_sharded_step_matches_one_gpu():
    from diffrast import _native
    from diffrast.scenes import config4_params

    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
        res = dict(out)
    assert res[0] == res[1]  # replicated parameters stay identical
    p = torch.from_numpy(config4_params(1024, 4000)).cuda()
    target = _native.render(torch.from_numpy(config4_params(1024, 4001)).cuda(), 512, 512, 0.0015)
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    for t in range(1, 4):
        losses, g = _native.loss_backward(p, target, 0.0015)
        _native.adam_step(p, m, v, g, t)
    np.testing.assert_allclose(res[0][0], losses.cpu().numpy(), rtol=1e-5)
    np.testing.assert_allclose(np.array(res[0][1]), p.cpu().numpy(), rtol=1e-4, atol=1e-6)
