"""Deterministic gradient sums (dr_set_deterministic).

With the setting on, per-warp gradient totals are added in 64-bit fixed
point, so the result does not depend on the order of the GPU's atomic
additions: repeated calls and repeated fits are bit-identical, and so are the
kernels that group the same warp blocks differently (region and tile kernels,
gathered and windowed lists). The values stay within the north star's
tolerance of the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_grads_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def native():
    from diffrast import _native

    assert torch.cuda.is_available(), "GPU tests need CUDA"
    _native.set_deterministic(True)
    yield _native
    _native.set_deterministic(False)


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def test_setting_round_trips(native):
    assert native.get_deterministic() is True
    L = native.lib()
    import ctypes

    dev = torch.device("cuda", 0)
    h = native.context(dev, torch.cuda.current_stream(dev).cuda_stream)
    on = ctypes.c_int(-1)
    native.check(L.dr_get_deterministic(h, ctypes.byref(on)))
    assert on.value == 1
    with pytest.raises(Exception):
        native.check(L.dr_set_deterministic(h, 2))


def test_headline_cell_repeats_bit_for_bit_and_matches_the_oracle(native, oracle):
    from diffrast.scenes import config2_params

    p, tp = config2_params(32, 128, 5)
    target = oracle.render_batch(tp, 256, 256, 0.0015)
    P, Tg = cuda(p), cuda(target)
    l1, g1 = native.loss_backward(P, Tg, 0.0015)
    l2, g2 = native.loss_backward(P, Tg, 0.0015)
    assert torch.equal(g1, g2) and torch.equal(l1, l2)
    _, ref_g = oracle.backward_batch(p, target, 0.0015)
    assert_grads_close(g1.cpu().numpy(), ref_g, "deterministic headline grads")
    # The region kernel (32 scenes) and the tile kernel (4-scene calls) reduce
    # the same warp blocks: their fixed-point sums are identical.
    assert native.query_path(32, 128, 256, 256) == native.PATH_REGION
    native.set_triangle_split(1)
    try:
        for lo in (0, 12, 28):
            assert native.query_path(4, 128, 256, 256) == native.PATH_TILE
            _, g4 = native.loss_backward(P[lo:lo + 4].contiguous(), Tg[lo:lo + 4].contiguous(),
                                         0.0015)
            assert torch.equal(g4, g1[lo:lo + 4])
    finally:
        native.set_triangle_split(0)


def test_gathered_and_windowed_lists_give_the_same_sums(native):
    from test_gpu_gather import clustered_scene

    T = 8192
    native.set_triangle_split(1)
    try:
        p = np.stack([clustered_scene(T, 9, clusters=5, spread=0.12, dead_every=13)])
        q = np.concatenate([p, np.zeros((1, 1, 10), np.float32)], axis=1)
        target = np.random.default_rng(3).uniform(0, 1, size=(1, 96, 96, 3)).astype(np.float32)
        _, gg = native.loss_backward(cuda(p), cuda(target), 0.002)
        _, gw = native.loss_backward(cuda(q), cuda(target), 0.002)
        assert torch.equal(gg, gw[:, :T])
        _, gg2 = native.loss_backward(cuda(p), cuda(target), 0.002)
        assert torch.equal(gg, gg2)
    finally:
        native.set_triangle_split(0)


@pytest.fixture
def no_split(native):
    # The triangle-block split composes each pixel's blocks, so its sums differ
    # (to rounding) from the unsplit kernels', and the automatic choice depends
    # on the batch: compare the unsplit kernels.
    native.set_triangle_split(1)
    yield
    native.set_triangle_split(0)


def test_upstream_gradient_and_host_buffer_calls_repeat(native, no_split):
    from diffrast.scenes import uniform_scenes

    p = uniform_scenes(6, 300, 17)
    g_in = np.random.default_rng(4).normal(0, 1e-3, size=(6, 80, 72, 3)).astype(np.float32)
    a = native.grad_backward(cuda(p), cuda(g_in), 0.003)
    b = native.grad_backward(cuda(p), cuda(g_in), 0.003)
    assert torch.equal(a, b)
    tgt = torch.from_numpy(np.random.default_rng(5).uniform(0, 1, (6, 80, 72, 3)).astype(
        np.float32)).pin_memory()
    pp = torch.from_numpy(p).pin_memory()
    l1, h1 = native.loss_backward_host(pp, tgt, 0.003)
    l2, h2 = native.loss_backward_host(pp, tgt, 0.003)
    assert torch.equal(h1, h2) and torch.equal(l1, l2)
    _, d1 = native.loss_backward(pp.cuda(), tgt.cuda(), 0.003)
    assert torch.equal(d1.cpu(), h1)  # chunked host pipeline: same sums


def test_fits_repeat_bit_for_bit(native):
    g = torch.Generator(device="cuda").manual_seed(8)
    target = torch.rand(48, 40, 3, device="cuda", generator=g)
    p = torch.rand(150, 10, device="cuda", generator=g) * 0.6 + 0.2
    a = native.fit(target, p, [0.3, 0.3, 0.3], iters=120, patience=None)
    b = native.fit(target.clone(), p.clone(), [0.3, 0.3, 0.3], iters=120, patience=None)
    assert torch.equal(a["losses"], b["losses"])
    assert torch.equal(a["final_params"], b["final_params"])
    assert torch.equal(a["best_params"], b["best_params"])
    assert a["best_loss"] == b["best_loss"]


def test_non_finite_totals_propagate_like_float_sums(native):
    # A NaN target pixel makes the gradient NaN for the triangles over it,
    # as the float sums do.
    from diffrast.scenes import uniform_scenes

    p = uniform_scenes(2, 40, 23)
    target = np.random.default_rng(6).uniform(0, 1, size=(2, 64, 64, 3)).astype(np.float32)
    target[1, 30:34, 30:34, :] = np.nan
    _, gd = native.loss_backward(cuda(p), cuda(target), 0.004)
    native.set_deterministic(False)
    try:
        _, gf = native.loss_backward(cuda(p), cuda(target), 0.004)
    finally:
        native.set_deterministic(True)
    assert torch.equal(torch.isnan(gd), torch.isnan(gf))
    assert torch.isnan(gd[1]).any() and not torch.isnan(gd[0]).any()
    ok = ~torch.isnan(gf)
    torch.testing.assert_close(gd[ok], gf[ok], rtol=1e-4, atol=1e-7)
