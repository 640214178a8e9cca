"""CUDA path vs the CPU oracle (the reference's algorithm restated), on the same
seeded inputs. Tolerances are the north star's: images |d| <= 1e-5 + 1e-4|ref|,
gradients per element |d| <= 1e-6 + 1e-3|ref|.

Every call goes through the C ABI (libdiffrast_cuda.so) via diffrast._native.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import (assert_grads_close, assert_images_close, rel_norm_error)

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def native():
    from diffrast import _native

    assert torch.cuda.is_available(), "GPU tests need CUDA"
    return _native


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def run_all(native, oracle, params, target, sigma, bg=(0.0, 0.0, 0.0), check_grads=True,
            slack=False):
    """Forward, loss+backward, grad-input backward; compare each to the oracle."""
    B, T = params.shape[:2]
    H, W = target.shape[1], target.shape[2]
    img = host(native.render(cuda(params), H, W, sigma, bg))
    ref_img = oracle.render_batch(params, H, W, sigma, bg)
    assert_images_close(img, ref_img, "render")

    losses, grads, img2 = native.loss_backward(cuda(params), cuda(target), sigma, bg,
                                               want_image=True)
    losses, grads, img2 = host(losses), host(grads), host(img2)
    ref_l, ref_g, ref_img2 = oracle.backward_batch(params, target, sigma, bg, want_images=True)
    assert_images_close(img2, ref_img2, "fused render")
    np.testing.assert_allclose(losses, ref_l, rtol=1e-5, atol=1e-9)
    if check_grads:
        sl = None
        if slack:
            _, g64 = oracle.backward_batch(params, target, sigma, bg, f64=True)
            sl = np.abs(ref_g.astype(np.float64) - g64)
        assert_grads_close(grads, ref_g, "loss grads", slack=sl)
        for b in range(B):
            assert rel_norm_error(grads[b], ref_g[b]) < 1e-3

    # Upstream-gradient mode (autograd path) vs the oracle's direct variant.
    g_in = np.random.default_rng(7).normal(0, 1e-4, size=target.shape).astype(np.float32)
    gg = host(native.grad_backward(cuda(params), cuda(g_in), sigma, bg))
    _, ref_gg = oracle.backward_batch(params, g_in, sigma, bg, mode=oracle.MODE_DIRECT_GRAD)
    if check_grads:
        sl = None
        if slack:
            _, g64 = oracle.backward_batch(params, g_in, sigma, bg, mode=oracle.MODE_DIRECT_GRAD,
                                           f64=True)
            sl = np.abs(ref_gg.astype(np.float64) - g64)
        assert_grads_close(gg, ref_gg, "grad-input grads", slack=sl)
    return img, grads


def tri(verts, color, alpha):
    return np.array(list(np.ravel(verts)) + list(color) + [alpha], dtype=np.float32)


def test_reference_test_scenes(native, oracle):
    # grad.rs:329-346 scene_pair at the sigmas its tests use.
    bg = (0.1, 0.12, 0.15)
    target_p = np.stack([
        tri([[0.25, 0.30], [0.80, 0.22], [0.55, 0.78]], [0.9, 0.3, 0.2], 0.8),
        tri([[0.15, 0.60], [0.70, 0.65], [0.40, 0.20]], [0.2, 0.6, 0.9], 0.6)])[None]
    scene = np.stack([
        tri([[0.21, 0.34], [0.77, 0.26], [0.58, 0.72]], [0.7, 0.4, 0.3], 0.7),
        tri([[0.18, 0.55], [0.66, 0.69], [0.44, 0.24]], [0.3, 0.5, 0.8], 0.5)])[None]
    for sigma in (0.01, 0.02, 0.03):
        target = oracle.render_batch(target_p, 48, 48, sigma, bg)
        run_all(native, oracle, scene, target, sigma, bg)


def test_unit_triangle_paints_over_background(native):
    # raster.rs:212-220 on the GPU.
    p = np.array([[[0.2, 0.2, 0.8, 0.2, 0.5, 0.8, 1.0, 0.0, 0.0, 1.0]]], np.float32)
    img = host(native.render(cuda(p), 64, 64, 0.002))[0]
    assert img[25, 32, 0] > 0.99 and img[25, 32, 1] < 0.01
    assert np.array_equal(img[63, 0], [0.0, 0.0, 0.0])


@pytest.mark.parametrize("W,H,T", [(37, 19, 33), (8, 8, 1), (17, 41, 65), (64, 64, 32),
                                   (96, 80, 200), (1, 1, 4), (64, 1, 8), (1, 64, 8)])
@pytest.mark.parametrize("sigma", [0.0015, 0.01, 0.03])
def test_seeded_scenes_match_oracle(native, oracle, W, H, T, sigma):
    from diffrast.scenes import uniform_scenes

    params = uniform_scenes(3, T, seed=W * 1000 + H * 10 + T)
    target = oracle.render_batch(uniform_scenes(3, T, seed=17 + T), H, W, sigma, (0.2, 0.3, 0.4))
    run_all(native, oracle, params, target, sigma, (0.05, 0.1, 0.15))


def test_small_triangles_like_reference_benches(native, oracle):
    # Scene::random(n, bg, 0.15) shapes (benches/raster.rs:16-19): small triangles.
    rng = np.random.default_rng(11)
    B, T = 4, 128
    c = rng.uniform(0, 1, size=(B, T, 1, 2))
    v = c + rng.uniform(-0.15, 0.15, size=(B, T, 3, 2))
    p = np.concatenate([v.reshape(B, T, 6), rng.uniform(0, 1, (B, T, 3)),
                        rng.uniform(0.3, 0.8, (B, T, 1))], -1).astype(np.float32)
    target = np.full((B, 64, 64, 3), 0.3, np.float32)
    run_all(native, oracle, p, target, 0.01, (0.5, 0.5, 0.5))


def test_layouts_agree(native):
    from diffrast.scenes import uniform_scenes

    p = cuda(uniform_scenes(2, 40, 3))
    a = native.render(p, 33, 47, 0.01, layout=native.LAYOUT_BHWC)
    b = native.render(p, 33, 47, 0.01, layout=native.LAYOUT_BCHW)
    assert torch.equal(a.permute(0, 3, 1, 2), b)
    tgt = torch.rand(2, 33, 47, 3, device="cuda")
    la, ga = native.loss_backward(p, tgt, 0.01, layout=native.LAYOUT_BHWC)
    lb, gb = native.loss_backward(p, tgt.permute(0, 3, 1, 2).contiguous(), 0.01,
                                  layout=native.LAYOUT_BCHW)
    assert torch.equal(la, lb)
    # Images and losses are bit-identical; gradients are sums of f32 atomics
    # whose order varies run to run (a few ulps of the largest term).
    torch.testing.assert_close(ga, gb, rtol=1e-5, atol=1e-8)


def test_many_triangles_span_several_bins(native, oracle):
    # More triangles than one shared-memory chunk holds, heavily overlapping.
    from diffrast.scenes import uniform_scenes

    p = uniform_scenes(2, 700, 5, lo=0.3, hi=0.7)
    target = oracle.render_batch(uniform_scenes(2, 50, 6), 40, 40, 0.005)
    run_all(native, oracle, p, target, 0.005)


def test_per_scene_backgrounds_and_order(native, oracle):
    from diffrast.scenes import uniform_scenes

    p = uniform_scenes(6, 5, 9)
    bgs = np.array([[i / 6.0] * 3 for i in range(6)], np.float32)
    target = np.random.default_rng(1).uniform(0, 1, (6, 16, 16, 3)).astype(np.float32)
    run_all(native, oracle, p, target, 0.02, bgs)


def test_empty_inputs(native):
    p = cuda(np.zeros((0, 4, 10)))
    assert native.render(p, 8, 8, 0.01).shape == (0, 8, 8, 3)
    img = host(native.render(cuda(np.zeros((2, 0, 10))), 16, 16, 0.01, (0.2, 0.4, 0.6)))
    assert np.all(img == np.array([0.2, 0.4, 0.6], np.float32))
    tgt = np.full((2, 16, 16, 3), 0.5, np.float32)
    l, g = native.loss_backward(cuda(np.zeros((2, 0, 10))), cuda(tgt), 0.01, (0.2, 0.4, 0.6))
    assert g.shape == (2, 0, 10)
    np.testing.assert_allclose(host(l), np.mean((img - 0.5) ** 2, axis=(1, 2, 3)), rtol=1e-6)


def test_edge_case_triangles(native, oracle):
    # Off-screen, zero / one / tiny / NaN opacity, coincident, collinear and
    # NaN-vertex triangles in one scene.
    rows = [
        tri([[5.0, 5.0], [6.0, 5.0], [5.5, 6.0]], [1, 1, 1], 1.0),
        tri([[0.1, 0.1], [0.9, 0.2], [0.4, 0.9]], [1, 0, 0], 0.0),
        tri([[0.2, 0.1], [0.8, 0.8], [0.1, 0.7]], [0, 1, 0], 1.0),
        tri([[0.3, 0.3], [0.6, 0.3], [0.45, 0.6]], [0, 0, 1], 5e-7),
        tri([[0.5, 0.5], [0.5, 0.5], [0.5, 0.5]], [1, 1, 0], 0.9),
        tri([[0.2, 0.2], [0.4, 0.4], [0.8, 0.8]], [0, 1, 1], 0.8),
        tri([[0.2, 0.6], [0.2, 0.6], [0.9, 0.1]], [1, 0, 1], 0.7),
        tri([[np.nan, 0.6], [0.2, 0.6], [0.9, 0.1]], [1, 0, 1], 0.7),
        tri([[0.0, 0.0], [1.0, 0.0], [0.0, 1.0]], [0.3, 0.3, 0.3], 1.0),
        tri([[0.3, 0.2], [0.7, 0.4], [0.5, 0.9]], [0.9, 0.1, 0.5], 0.6),
    ]
    p = np.stack(rows)[None]
    target = np.random.default_rng(3).uniform(0, 1, (1, 32, 32, 3)).astype(np.float32)
    for sigma in (0.001, 0.02):
        run_all(native, oracle, p, target, sigma, (0.1, 0.2, 0.3))
        _, g = oracle.backward_batch(p, target, sigma)
        assert g[0, 2, 9] == 0.0  # alpha == 1 is pinned (grad.rs:471-481)


def test_nan_alpha_render_vs_tape_semantics(native, oracle):
    # raster::render paints a NaN-alpha triangle (alpha <= 0 is false) while
    # render_with_tape drops it (alpha > 0 is false); both paths must agree.
    p = np.stack([tri([[0.1, 0.1], [0.9, 0.2], [0.4, 0.9]], [1, 0, 0], 0.5),
                  tri([[0.3, 0.3], [0.7, 0.3], [0.5, 0.7]], [0, 1, 0], np.nan)])[None]
    img = host(native.render(cuda(p), 24, 24, 0.01))
    ref = oracle.render_batch(p, 24, 24, 0.01)
    assert np.isnan(ref).any()
    assert_images_close(img, ref, "NaN-alpha render")
    target = np.zeros((1, 24, 24, 3), np.float32)
    l, g, im2 = native.loss_backward(cuda(p), cuda(target), 0.01, want_image=True)
    rl, rg, rim = oracle.backward_batch(p, target, 0.01, want_images=True)
    assert not np.isnan(rim).any()
    assert_images_close(host(im2), rim, "NaN-alpha taped render")
    assert_grads_close(host(g), rg)


@pytest.mark.parametrize("sigma", [0.00015, 0.0015, 0.015])
def test_config5_stress(native, oracle, sigma):
    from diffrast.scenes import config5_params

    p = config5_params(2, 2048, 5000)
    target = oracle.render_batch(config5_params(2, 2048, 5100), 512, 512, sigma)
    img, grads = run_all(native, oracle, p, target, sigma)
    assert np.isfinite(img).all() and np.isfinite(grads).all()
    zero_alpha = p[..., 9] == 0.0
    assert np.all(grads[zero_alpha] == 0.0)
    one_alpha = p[..., 9] == 1.0
    assert np.all(grads[one_alpha][:, 9] == 0.0)


def test_config4_large_scene(native, oracle):
    from diffrast.scenes import config4_params

    p = config4_params(4096, 4000)
    target = oracle.render_batch(config4_params(4096, 4001), 1024, 1024, 0.0015)
    run_all(native, oracle, p, target, 0.0015)


@pytest.mark.parametrize("T", [32, 128, 512])
@pytest.mark.parametrize("size", [64, 128, 256])
def test_config2_cells(native, oracle, T, size):
    from diffrast.scenes import config2_params

    cell = [32, 128, 512].index(T) * 3 + [64, 128, 256].index(size)
    p, tp = config2_params(4, T, cell)
    target = oracle.render_batch(tp, size, size, 0.0015)
    run_all(native, oracle, p, target, 0.0015)


def test_headline_batch_properties(native):
    # Full B=32, T=128, 256^2: the batch result equals each scene run alone,
    # and the fused loss equals the MSE of the fused render.
    from diffrast.scenes import config2_params

    p, tp = config2_params(32, 128, 5)
    P, TP = cuda(p), cuda(tp)
    tgt = native.render(TP, 256, 256, 0.0015)
    losses, grads, img = native.loss_backward(P, tgt, 0.0015, want_image=True)
    for b in (0, 17, 31):
        # A scene alone has too few tiles to fill the GPU and would take the
        # triangle split, which rounds the composite differently: compare the
        # unsplit path bitwise, the split one to rounding.
        native.set_triangle_split(1)
        try:
            lb, gb, ib = native.loss_backward(P[b:b + 1], tgt[b:b + 1], 0.0015, want_image=True)
        finally:
            native.set_triangle_split(0)
        assert torch.equal(ib[0], img[b])
        assert lb[0].item() == losses[b].item()
        # f32 atomic accumulation order varies run to run: a few ulps.
        torch.testing.assert_close(gb[0], grads[b], rtol=1e-5, atol=1e-8)
        ls, gs, is_ = native.loss_backward(P[b:b + 1], tgt[b:b + 1], 0.0015, want_image=True)
        torch.testing.assert_close(is_[0], img[b], rtol=0, atol=2e-6)
        torch.testing.assert_close(ls[0], losses[b], rtol=1e-6, atol=0)
        assert_grads_close(host(gs[0]), host(grads[b]), "split single scene")
    mse = ((img.double() - tgt.double()) ** 2).flatten(1).mean(1)
    torch.testing.assert_close(losses.double(), mse, rtol=1e-6, atol=0)
    assert torch.isfinite(grads).all()


def test_mse_kernel_matches_oracle(native, oracle):
    rng = np.random.default_rng(0)
    a = rng.uniform(0, 1, (3, 192, 192, 3)).astype(np.float32)
    b = rng.uniform(0, 1, (3, 192, 192, 3)).astype(np.float32)
    got = host(native.mse_loss(cuda(a), cuda(b)))
    for i in range(3):
        assert abs(got[i] - oracle.mse(a[i], b[i])) <= 1e-7 * abs(got[i])


@pytest.mark.parametrize("shape", [(1, 1, 1, 3), (4, 5, 7, 3), (2, 301, 257, 3), (40, 64, 64, 3)])
def test_mse_kernel_sizes_and_determinism(native, oracle, shape):
    # One chunk, many chunks with a ragged last chunk, and many images; the
    # chunk partials are summed in a fixed order, so repeated calls agree bitwise.
    rng = np.random.default_rng(sum(shape))
    a = rng.uniform(-1, 2, shape).astype(np.float32)
    b = rng.uniform(-1, 2, shape).astype(np.float32)
    first = host(native.mse_loss(cuda(a), cuda(b)))
    again = host(native.mse_loss(cuda(a), cuda(b)))
    assert np.array_equal(first, again)
    ref = np.array([oracle.mse(a[i], b[i]) for i in range(shape[0])], np.float32)
    np.testing.assert_allclose(first, ref, rtol=1e-7, atol=0)


@pytest.mark.parametrize("tris", [97, 96])  # scalar kernel (n % 4 != 0) and the float4 kernel
def test_adam_is_bit_exact(native, oracle, tris):
    rng = np.random.default_rng(4)
    n = 10 * tris
    p0 = rng.uniform(-0.5, 1.5, n).astype(np.float32)
    p0[5] = np.nan
    lr = oracle.learning_rates(tris)
    adam = oracle.Adam(n)
    p_ref = p0.copy()
    P, M, V = cuda(p0), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    for step in range(1, 30):
        g = rng.normal(0, 1e-2, n).astype(np.float32)
        adam.step(p_ref, g, lr)
        oracle.project(p_ref)
        native.adam_step(P, M, V, cuda(g), step)
        assert np.array_equal(host(P), p_ref, equal_nan=True), step


@pytest.fixture()
def strict(native):
    native.set_precision(native.PRECISION_STRICT)
    yield
    native.set_precision(native.PRECISION_REFERENCE)


@pytest.mark.parametrize("W,H,T", [(37, 19, 33), (64, 64, 32), (96, 80, 200)])
def test_strict_mode_matches_oracle(native, oracle, strict, W, H, T):
    from diffrast.scenes import uniform_scenes

    params = uniform_scenes(2, T, seed=W + H + T)
    target = oracle.render_batch(uniform_scenes(2, T, seed=99), H, W, 0.01)
    run_all(native, oracle, params, target, 0.01)


def test_strict_and_default_modes_agree(native, oracle):
    from diffrast.scenes import config2_params

    p, tp = config2_params(4, 128, 5)
    P = cuda(p)
    tgt = native.render(cuda(tp), 128, 128, 0.0015)
    lf, gf, imf = native.loss_backward(P, tgt, 0.0015, want_image=True)
    native.set_precision(native.PRECISION_STRICT)
    try:
        ls, gs, ims = native.loss_backward(P, tgt, 0.0015, want_image=True)
    finally:
        native.set_precision(native.PRECISION_REFERENCE)
    assert_images_close(host(imf), host(ims), "default vs strict render")
    np.testing.assert_allclose(host(lf), host(ls), rtol=1e-5)
    assert_grads_close(host(gf), host(gs), "default vs strict grads")


@pytest.mark.parametrize("size,T,sigma", [(64, 32, 0.0015), (128, 128, 0.0015), (96, 200, 0.01)])
def test_fast_mode_tracks_the_exact_gradient(native, oracle, size, T, sigma):
    # DR_PRECISION_FAST skips the reference's f32 cancellation near edges, so it
    # is judged against the f64 twin, with the f32 reference's own distance
    # from it as the allowance.
    from diffrast.scenes import uniform_scenes

    p = uniform_scenes(3, T, 40 + T)
    target = oracle.render_batch(uniform_scenes(3, T, 41 + T), size, size, sigma)
    native.set_precision(native.PRECISION_FAST)
    try:
        l, g, im = native.loss_backward(cuda(p), cuda(target), sigma, want_image=True)
    finally:
        native.set_precision(native.PRECISION_REFERENCE)
    l32, g32, im32 = oracle.backward_batch(p, target, sigma, want_images=True)
    l64, g64, im64 = oracle.backward_batch(p, target, sigma, f64=True, want_images=True)
    assert_images_close(host(im), im64, "fast render vs f64")
    np.testing.assert_allclose(host(l), l64, rtol=1e-5)
    assert_grads_close(host(g), g64, "fast grads vs f64", slack=np.abs(g32 - g64))


@pytest.mark.parametrize("B,per_scene_bg,layout", [(7, False, 0), (32, True, 0), (5, True, 1)])
def test_host_buffers_pipelined_equal_device_path(native, B, per_scene_bg, layout):
    # Host tensors take the library's chunked upload/compute/download pipeline
    # (dr_loss_backward_host) and come back as host tensors; results equal the
    # device-tensor call. Chunks of a few scenes may take the triangle split
    # while the whole batch does not, so the two agree to rounding.
    from diffrast.scenes import uniform_scenes

    p = torch.from_numpy(uniform_scenes(B, 48, 11)).pin_memory()
    tgt = torch.rand(B, 40, 52, 3, generator=torch.Generator().manual_seed(1))
    if layout == native.LAYOUT_BCHW:
        tgt = tgt.permute(0, 3, 1, 2).contiguous()
    tgt = tgt.pin_memory()
    bg = (torch.rand(B, 3, generator=torch.Generator().manual_seed(2)) if per_scene_bg
          else (0.1, 0.2, 0.3))
    l_h, g_h = native.loss_backward(p, tgt, 0.004, bg, layout=layout)
    assert not l_h.is_cuda and not g_h.is_cuda and l_h.is_pinned() and g_h.is_pinned()
    l_d, g_d = native.loss_backward(p.cuda(), tgt.cuda(), 0.004, bg, layout=layout)
    torch.testing.assert_close(l_h, l_d.cpu(), rtol=1e-6, atol=0)
    assert_grads_close(host(g_h), host(g_d), "host pipeline")
    # Pageable buffers take the same path through the driver's staging.
    l_p, g_p = native.loss_backward_host(p.clone(), tgt.clone(), 0.004, bg, layout=layout)
    assert not l_p.is_pinned()
    torch.testing.assert_close(l_p, l_h, rtol=0, atol=0)
    assert_grads_close(host(g_p), host(g_h), "pageable host buffers")


@pytest.mark.parametrize("B,T", [(1, 40), (3, 0), (2, 130)])
def test_host_buffers_single_scene_empty_and_long_lists(native, B, T):
    # dr_loss_backward_host on one scene (one chunk, which may take the
    # triangle split), on scenes without triangles (loss of the background
    # alone), and on lists longer than one binning chunk (tile kernel).
    from diffrast.scenes import uniform_scenes

    p = torch.from_numpy(uniform_scenes(B, T, 21)).pin_memory() if T else \
        torch.zeros(B, 0, 10).pin_memory()
    tgt = torch.rand(B, 33, 47, 3, generator=torch.Generator().manual_seed(3)).pin_memory()
    l_h, g_h = native.loss_backward_host(p, tgt, 0.004, (0.3, 0.2, 0.1))
    l_d, g_d = native.loss_backward(p.cuda(), tgt.cuda(), 0.004, (0.3, 0.2, 0.1))
    torch.testing.assert_close(l_h, l_d.cpu(), rtol=1e-6, atol=0)
    assert g_h.shape == (B, T, 10)
    if T:
        assert_grads_close(host(g_h), host(g_d), "host buffers")


@pytest.fixture(params=[1, 2, 3, 8])
def split(native, request):
    native.set_triangle_split(request.param)
    yield request.param
    native.set_triangle_split(0)


def test_triangle_split_matches_oracle(native, oracle, split):
    # The triangle-block split (forward per block, per-pixel combine of the
    # blocks' maps, gradient per block) against the oracle, forced to 1, 2, 3
    # and 8 blocks: opaque and NaN-alpha layers, degenerate and coincident
    # triangles (a config 5 crop), per-scene backgrounds, ragged sizes.
    from diffrast.scenes import config5_params, uniform_scenes

    p = np.concatenate([uniform_scenes(2, 96, 71), config5_params(2, 96, 5200)], axis=0)
    p[0, 10, 9] = 1.0   # opaque: nothing beneath gets gradient at covered pixels
    p[0, 50, 9] = 1.0
    p[1, 20, 9] = np.nan  # the tape drops it (grad.rs:62)
    bg = np.random.default_rng(3).uniform(0, 1, (4, 3)).astype(np.float32)
    tp = uniform_scenes(4, 60, 72)
    target = oracle.render_batch(tp, 37, 45, 0.004, bg)
    run_all(native, oracle, p, target, 0.004, bg)


def test_fit_with_triangle_split_matches_unsplit(native, split):
    # dr_fit's graph takes the split path for small single scenes.
    from diffrast.scenes import config1_target_scene, seed_scene_geometry

    tgt = native.render(cuda(config1_target_scene(100, 0)), 64, 64, 0.0015)[0]
    init = torch.from_numpy(seed_scene_geometry(100, 1))
    init[:, 6:9] = 0.5
    r = native.fit(tgt, init, (0.2, 0.2, 0.2), 40)
    native.set_triangle_split(1)
    ref = native.fit(tgt, init, (0.2, 0.2, 0.2), 40)
    np.testing.assert_allclose(host(r["losses"]), host(ref["losses"]), rtol=2e-4)


def test_region_kernel_bchw_and_per_scene_backgrounds(native, oracle):
    # B=32 at 256^2 with T <= 128 takes the region kernel (2x2 tiles per CTA,
    # blocks taken from a shared counter, centre-out launch order); here with
    # the torch (B, 3, H, W) layout, one background per scene and the
    # upstream-gradient mode, against the oracle on every scene.
    from diffrast.scenes import uniform_scenes

    B, T, H, W = 32, 48, 256, 256
    p = uniform_scenes(B, T, 81)
    bg = np.random.default_rng(5).uniform(0, 1, (B, 3)).astype(np.float32)
    tgt = oracle.render_batch(uniform_scenes(B, T, 82), H, W, 0.0015, bg)
    t_bchw = np.ascontiguousarray(tgt.transpose(0, 3, 1, 2))
    losses, grads, img = native.loss_backward(cuda(p), cuda(t_bchw), 0.0015, bg,
                                              layout=native.LAYOUT_BCHW, want_image=True)
    ref_l, ref_g, ref_img = oracle.backward_batch(p, tgt, 0.0015, bg, want_images=True)
    assert_images_close(host(img).transpose(0, 2, 3, 1), ref_img, "region BCHW image")
    np.testing.assert_allclose(host(losses), ref_l, rtol=1e-5, atol=1e-9)
    assert_grads_close(host(grads), ref_g, "region BCHW grads")
    g_in = np.random.default_rng(6).normal(0, 1e-4, size=(B, 3, H, W)).astype(np.float32)
    gg = host(native.grad_backward(cuda(p), cuda(g_in), 0.0015, bg, layout=native.LAYOUT_BCHW))
    _, ref_gg = oracle.backward_batch(p, np.ascontiguousarray(g_in.transpose(0, 2, 3, 1)), 0.0015,
                                      bg, mode=oracle.MODE_DIRECT_GRAD)
    assert_grads_close(gg, ref_gg, "region BCHW grad-input")
