"""The tile kernel's gathered lists (128 < T <= 8192) against the oracle and
against the fixed-window lists.

A CTA marks, one bit per triangle, the live triangles whose pixel boxes meet
its tile, and takes its lists from the marked ones in triangle order, cut at
exactly 128 (mid-word when a word overfills a list). The composite must run
over the same sequence as the fixed 128-triangle windows give, so images are
bit-identical between the two forms and gradients agree to rounding.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_grads_close, assert_images_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def native():
    from diffrast import _native

    assert torch.cuda.is_available(), "GPU tests need CUDA"
    _native.set_triangle_split(1)  # the split path would take these small batches
    yield _native
    _native.set_triangle_split(0)


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def clustered_scene(T, seed, clusters=3, spread=0.08, dead_every=0):
    """Small triangles around a few centres: most tiles see few of them, a
    few tiles see many (lists cut mid-word), some tiles none."""
    rng = np.random.default_rng(seed)
    centres = rng.uniform(0.15, 0.85, size=(clusters, 2))
    c = centres[rng.integers(0, clusters, size=T)] + rng.normal(0, spread, size=(T, 2))
    v = c[:, None, :] + rng.uniform(-0.04, 0.04, size=(T, 3, 2))
    p = np.empty((T, 10), np.float32)
    p[:, :6] = v.reshape(T, 6)
    p[:, 6:9] = rng.uniform(0, 1, size=(T, 3))
    p[:, 9] = rng.uniform(0.2, 0.9, size=T)
    if dead_every:
        p[::dead_every, 9] = 0.0              # alpha 0: never marked
        p[1::dead_every * 2, 0] = np.nan      # no pixel box: never marked
        p[2::dead_every * 3, 9] = 1.0         # opaque
    return p


@pytest.mark.parametrize("T,size", [(129, 64), (300, 96), (1000, 128), (4096, 160)])
def test_gathered_lists_match_the_oracle(native, oracle, T, size):
    p = np.stack([clustered_scene(T, 11 + T), clustered_scene(T, 12 + T, dead_every=7)])
    target = oracle.render_batch(np.stack([clustered_scene(T, 13 + T)] * 2), size, size, 0.002)
    assert native.query_path(2, T, size, size) == native.PATH_TILE_GATHER
    img = host(native.render(cuda(p), size, size, 0.002, (0.1, 0.2, 0.3)))
    assert_images_close(img, oracle.render_batch(p, size, size, 0.002, (0.1, 0.2, 0.3)),
                        "gathered render")
    losses, grads, img2 = native.loss_backward(cuda(p), cuda(target), 0.002, (0.1, 0.2, 0.3),
                                               want_image=True)
    rl, rg, rimg = oracle.backward_batch(p, target, 0.002, (0.1, 0.2, 0.3), want_images=True)
    assert_images_close(host(img2), rimg, "gathered fused render")
    np.testing.assert_allclose(host(losses), rl, rtol=1e-5, atol=1e-9)
    assert_grads_close(host(grads), rg, "gathered loss grads")
    g_in = np.random.default_rng(T).normal(0, 1e-4, size=target.shape).astype(np.float32)
    gg = host(native.grad_backward(cuda(p), cuda(g_in), 0.002, (0.1, 0.2, 0.3)))
    _, ref_gg = oracle.backward_batch(p, g_in, 0.002, (0.1, 0.2, 0.3),
                                      mode=oracle.MODE_DIRECT_GRAD)
    assert_grads_close(gg, ref_gg, "gathered grad-input grads")


def test_gathered_and_windowed_lists_composite_the_same_sequence(native):
    # 8192 triangles take the gathered form; one more (a dead triangle at the
    # end, alpha 0) takes the fixed windows. Same composite sequence: the images
    # and losses are bit-identical, the gradients equal to rounding.
    T = 8192
    p = np.stack([clustered_scene(T, 5, clusters=6, spread=0.15, dead_every=11)])
    q = np.concatenate([p, np.zeros((1, 1, 10), np.float32)], axis=1)
    assert native.query_path(1, T, 128, 128) == native.PATH_TILE_GATHER
    assert native.query_path(1, T + 1, 128, 128) == native.PATH_TILE
    target = np.random.default_rng(6).uniform(0, 1, size=(1, 128, 128, 3)).astype(np.float32)
    lg, gg, ig = native.loss_backward(cuda(p), cuda(target), 0.0015, want_image=True)
    lw, gw, iw = native.loss_backward(cuda(q), cuda(target), 0.0015, want_image=True)
    assert torch.equal(ig, iw) and torch.equal(lg, lw)
    torch.testing.assert_close(gg, gw[:, :T], rtol=1e-4, atol=1e-7)
    assert torch.count_nonzero(gw[:, T:]) == 0
    assert torch.equal(native.render(cuda(p), 128, 128, 0.0015),
                       native.render(cuda(q), 128, 128, 0.0015))


def test_tiles_no_triangle_reaches_still_report_their_loss(native, oracle):
    # Every triangle in the top-left corner: most tiles mark nothing, run no
    # list at all, and still add their pixels' squared error to the loss.
    T = 400
    p = clustered_scene(T, 21, clusters=1, spread=0.01)
    p[:, :6] = p[:, :6] * 0.2
    p = p[None]
    target = np.random.default_rng(22).uniform(0, 1, size=(1, 96, 96, 3)).astype(np.float32)
    losses, grads = native.loss_backward(cuda(p), cuda(target), 0.002, (0.5, 0.5, 0.5))
    rl, rg = oracle.backward_batch(p, target, 0.002, (0.5, 0.5, 0.5))
    np.testing.assert_allclose(host(losses), rl, rtol=1e-5)
    assert_grads_close(host(grads), rg, "corner scene grads")
