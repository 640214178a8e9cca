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

    def fake(params, targets, sigma, shard, n_shards, background=(0.0, 0.0, 0.0), out=None):
        # Partial results depend on the shard, like the kernel's, written into
        # the step's buffers as the kernel writes them.
        grads, sums = out
        grads.copy_(torch.full(params.shape, float(shard + 1)) *
                    torch.arange(params.numel()).reshape(params.shape))
        sums.fill_(10.0 * (shard + 1))
        return sums, grads

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
    g = step.loss_and_grads(target, 0.0015)[1].clone()  # the step reuses its buffer
    hist = [step.step(target, 0.0015).cpu().tolist() for _ in range(3)]
    torch.cuda.synchronize()
    out[rank] = (hist, step.params.cpu().numpy().tolist(), g.cpu().numpy().tolist())
    dist.destroy_process_group()


def _check_against_one_gpu(res, p, target):
    """Three single-GPU steps of loss_backward + Adam from the same start.

    The first gradient matches to the parity tolerance. Adam normalises each
    update, so a gradient that differs by rounding near zero can move its
    parameter by up to one learning rate more or less; the parameters after
    three steps must match closely except on such rare elements, and those stay
    within the step bound 2 x lr x steps."""
    from diffrast import _native

    m, v = torch.zeros_like(p), torch.zeros_like(p)
    hist = []
    for t in range(1, 4):
        losses, g = _native.loss_backward(p, target, 0.0015)
        if t == 1:
            assert_grads_close(np.array(res[2], np.float32), g.cpu().numpy(), "first gradient")
        hist.append(losses.cpu().tolist())
        _native.adam_step(p, m, v, g, t)
    np.testing.assert_allclose(np.array(res[0]), np.array(hist), rtol=1e-5)
    got, ref = np.array(res[1], np.float32), p.cpu().numpy()
    off = np.abs(got - ref) > 1e-6 + 1e-4 * np.abs(ref)
    assert off.mean() < 1e-3, f"{off.sum()} of {off.size} parameters differ"
    assert np.all(np.abs(got - ref) <= 2 * 0.02 * 3 + 1e-6)


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
    _check_against_one_gpu(res[0], p, target)


# ---- triangle-block sharding (TriangleShardedStep) --------------------------


def test_triangle_blocks_cover_every_triangle_once():
    from diffrast.sharded import triangle_block

    for T in (0, 1, 5, 63, 64, 150, 1000):
        for n in (1, 2, 3, 4, 8):
            got = [t for k in range(n) for t in range(*triangle_block(T, n, k))]
            assert got == list(range(T)), (T, n)
    with pytest.raises(ValueError):
        triangle_block(10, 2, 2)


def _gloo_block_worker(rank, world, port, out):
    import sys

    for p in (REPO, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    from diffrast import _native, sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)

    def fake_state(params, h, w, n_blocks):
        return torch.zeros(n_blocks, params.shape[0], h, w, 8)

    def fake_forward(params, h, w, sigma, n_blocks, block, state, background=(0.0, 0.0, 0.0)):
        # Only the own slice is written, like the kernel.
        state[block] = float(block + 1)

    def fake_backward(params, state, other, sigma, n_blocks, block, background=(0.0, 0.0, 0.0)):
        # The loss depends on every block's slice; the gradient only on the own block.
        loss = torch.tensor([float(state.sum())])
        g = torch.zeros_like(params)
        t0, t1 = sharded.triangle_block(params.shape[1], n_blocks, block)
        g[:, t0:t1] = float(block + 1)
        return loss, g

    def fake_adam(params, m, v, grads, step, *lrs):
        params -= grads

    _native.triangle_block_state = fake_state
    _native.triangle_block_forward = fake_forward
    _native.triangle_block_backward = fake_backward
    _native.adam_step = fake_adam
    step = sharded.TriangleShardedStep(torch.zeros(1, 5, 10))
    losses = step.step(torch.zeros(1, 2, 2, 3), 0.01)
    full = step.gather_params()
    out[rank] = (losses.tolist(), step.params.reshape(-1).tolist(), full.reshape(-1).tolist())
    dist.destroy_process_group()


def test_triangle_block_plumbing_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_gloo_block_worker, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        res = dict(out)
    # Both ranks combine the same gathered state: (1 + 2) * 2*2*8 per slice.
    assert res[0][0] == res[1][0] == [float((1 + 2) * 2 * 2 * 8)]
    own0 = np.array(res[0][1]).reshape(5, 10)
    own1 = np.array(res[1][1]).reshape(5, 10)
    assert np.all(own0[:3] == -1.0) and np.all(own0[3:] == 0.0)  # blocks [0,3) and [3,5)
    assert np.all(own1[:3] == 0.0) and np.all(own1[3:] == -2.0)
    full = np.array(res[0][2]).reshape(5, 10)
    assert np.array_equal(full, np.array(res[1][2]).reshape(5, 10))
    assert np.all(full[:3] == -1.0) and np.all(full[3:] == -2.0)


@pytest.mark.gpu
@pytest.mark.parametrize("n_blocks", [1, 2, 3, 4])
def test_triangle_blocks_emulated_on_one_gpu_match_the_oracle(oracle, n_blocks):
    # Every rank's calls run here in turn on one GPU: forward of each block
    # into its slice of the state, then the backward of each block. Every
    # block's call gives the same image and losses; the blocks' gradients sum
    # to the whole scene's. Opaque and NaN-alpha layers, per-scene backgrounds,
    # a ragged canvas.
    from diffrast import _native
    from diffrast.scenes import config5_params, uniform_scenes

    from conftest import assert_images_close

    p = np.concatenate([uniform_scenes(2, 96, 91), config5_params(1, 96, 5201)], axis=0)
    p[0, 10, 9] = 1.0
    p[1, 70, 9] = np.nan
    bg = np.random.default_rng(8).uniform(0, 1, (3, 3)).astype(np.float32)
    H, W, sigma = 37, 45, 0.004
    target = oracle.render_batch(uniform_scenes(3, 60, 92), H, W, sigma, bg)
    ref_l, ref_g, ref_img = oracle.backward_batch(p, target, sigma, bg, want_images=True)
    pc, tc = torch.from_numpy(p).cuda(), torch.from_numpy(target).cuda()
    state = _native.triangle_block_state(pc, H, W, n_blocks)
    for k in range(n_blocks):
        _native.triangle_block_forward(pc, H, W, sigma, n_blocks, k, state, bg)
    total = np.zeros_like(ref_g)
    first = None
    for k in range(n_blocks):
        losses, g, img = _native.triangle_block_backward(pc, state, tc, sigma, n_blocks, k, bg,
                                                         want_image=True)
        losses, g, img = losses.cpu().numpy(), g.cpu().numpy(), img.cpu().numpy()
        if first is None:
            first = (losses, img)
        else:  # the combine is the same computation on every rank
            assert np.array_equal(losses, first[0]) and np.array_equal(img, first[1])
        t0, t1 = (lambda per: (min(96, k * per), min(96, k * per + per)))(-(-96 // n_blocks))
        assert not np.any(g[:, :t0]) and not np.any(g[:, t1:])
        total += g
    assert_images_close(first[1], ref_img, "triangle-block image")
    np.testing.assert_allclose(first[0], ref_l, rtol=1e-5, atol=1e-9)
    assert_grads_close(total, ref_g, "triangle-block grads")
    # Upstream-gradient mode.
    g_in = np.random.default_rng(9).normal(0, 1e-4, size=target.shape).astype(np.float32)
    _, ref_gg = oracle.backward_batch(p, g_in, sigma, bg, mode=oracle.MODE_DIRECT_GRAD)
    gg = sum(_native.triangle_block_backward(pc, state, torch.from_numpy(g_in).cuda(), sigma,
                                             n_blocks, k, bg, grad_input=True)[1].cpu().numpy()
             for k in range(n_blocks))
    assert_grads_close(gg, ref_gg, "triangle-block grad-input")


def _nccl_block_worker(rank, world, port, out):
    import sys

    for p in (REPO, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist

    from diffrast import _native, sharded
    from diffrast.scenes import config1_target_scene, seed_scene_geometry

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    target = _native.render(torch.from_numpy(config1_target_scene(256, 0)).cuda(), 96, 96, 0.0015)
    p = torch.from_numpy(seed_scene_geometry(256, 1))[None].cuda()
    p[:, :, 6:9] = 0.5
    step = sharded.TriangleShardedStep(p)
    _, g = step.loss_and_grads(target, 0.0015)
    dist.all_reduce(g)  # the blocks' gradients are disjoint
    hist = [step.step(target, 0.0015).cpu().tolist() for _ in range(3)]
    full = step.gather_params()
    torch.cuda.synchronize()
    out[rank] = (hist, full.cpu().numpy().tolist(), g.cpu().numpy().tolist())
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_gpu_triangle_sharded_step_matches_one_gpu():
    from diffrast import _native
    from diffrast.scenes import config1_target_scene, seed_scene_geometry

    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_nccl_block_worker, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
        res = dict(out)
    assert res[0] == res[1]  # same losses and assembled parameters on both ranks
    target = _native.render(torch.from_numpy(config1_target_scene(256, 0)).cuda(), 96, 96, 0.0015)
    p = torch.from_numpy(seed_scene_geometry(256, 1))[None].cuda()
    p[:, :, 6:9] = 0.5
    _check_against_one_gpu(res[0], p, target)


def _leaving_worker(rank, world, port, out):
    import datetime
    import sys
    import time

    for p in (REPO, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    from diffrast import _native, sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))

    def fake(params, targets, sigma, shard, n_shards, background=(0.0, 0.0, 0.0), out=None):
        grads, sums = out
        grads.fill_(float(shard + 1))
        sums.fill_(1.0)
        return sums, grads

    _native.loss_backward_sharded = fake
    _native.adam_step = lambda *a, **k: None
    step = sharded.ShardedSceneStep(torch.zeros(1, 3, 10))
    tgt = torch.zeros(1, 4, 4, 3)
    step.step(tgt, 0.01)  # step 1: both ranks
    if rank == 1:
        out[1] = "left"
        os._exit(0)  # leaves between steps: no more collectives, no teardown
    t0 = time.monotonic()
    try:
        step.step(tgt, 0.01)  # step 2: the peer is gone
        out[0] = ("no error", time.monotonic() - t0)
    except Exception as e:  # the collective ends with an error
        out[0] = (type(e).__name__, time.monotonic() - t0)
    os._exit(0)


def test_a_departed_peer_ends_the_next_step_with_an_error():
    # Failure detection on the host: a rank that leaves between steps
    # (no kernel or collective of its own in flight) must make the others'
    # next collective fail within the process group's timeout, not hang.
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(90)
            assert p.exitcode == 0
        assert out[1] == "left"
        kind, waited = out[0]
    assert kind != "no error"
    assert waited < 30.0
