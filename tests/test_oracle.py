"""Pins the CPU oracle to the reference's own known-answer tests.

The reference ships no stored output vectors for this path; its behaviour is
pinned by unit and integration tests. Each test below restates one of them
(cited by file:line) against the oracle, which must pass all of them before it
is trusted as the parity checker.
"""

from __future__ import annotations

import numpy as np
import pytest

UNIT_TRI = [0.2, 0.2, 0.8, 0.2, 0.5, 0.8, 1.0, 0.0, 0.0, 1.0]  # raster.rs:174-176


def tri(verts, color, alpha):
    return np.array(list(np.ravel(verts)) + list(color) + [alpha], dtype=np.float32)


def scene_pair():
    """grad.rs:329-346: (scene params, target params, background)."""
    bg = (0.1, 0.12, 0.15)
    target = np.stack([
        tri([[0.25, 0.30], [0.80, 0.22], [0.55, 0.78]], [0.9, 0.3, 0.2], 0.8),
        tri([[0.15, 0.60], [0.70, 0.65], [0.40, 0.20]], [0.2, 0.6, 0.9], 0.6),
    ])
    scene = np.stack([
        tri([[0.21, 0.34], [0.77, 0.26], [0.58, 0.72]], [0.7, 0.4, 0.3], 0.7),
        tri([[0.18, 0.55], [0.66, 0.69], [0.44, 0.24]], [0.3, 0.5, 0.8], 0.5),
    ])
    return scene, target, bg


def reference_scene():
    """tests/integration.rs:12-17."""
    bg = (0.10, 0.11, 0.14)
    s = np.stack([
        tri([[0.20, 0.25], [0.80, 0.30], [0.50, 0.80]], [0.90, 0.30, 0.20], 0.9),
        tri([[0.30, 0.55], [0.85, 0.60], [0.60, 0.15]], [0.20, 0.60, 0.90], 0.7),
    ])
    return s, bg


def fit_target_scene():
    """fit.rs:431-440."""
    bg = (0.08, 0.09, 0.12)
    s = np.stack([
        tri([[0.20, 0.25], [0.80, 0.30], [0.50, 0.80]], [0.90, 0.30, 0.20], 0.9),
        tri([[0.30, 0.55], [0.85, 0.60], [0.60, 0.15]], [0.20, 0.60, 0.90], 0.7),
    ])
    return s, bg


# --- raster.rs:178-240 -----------------------------------------------------


def test_centroid_is_inside_and_far_corner_is_outside(oracle):
    t = np.array(UNIT_TRI, np.float32)
    assert oracle.signed_distance(t[:6], (0.5, 0.4)) > 0.0
    assert oracle.signed_distance(t[:6], (0.0, 0.0)) < 0.0


def test_coverage_is_half_on_the_edge(oracle):
    c = oracle.coverage(np.array(UNIT_TRI, np.float32), (0.5, 0.2), 0.01)
    assert abs(c - 0.5) < 1e-4


def test_coverage_saturates_away_from_the_edge(oracle):
    t = np.array(UNIT_TRI, np.float32)
    assert oracle.coverage(t, (0.5, 0.4), 0.002) > 0.999
    assert oracle.coverage(t, (0.02, 0.98), 0.002) < 1e-3


def test_winding_order_does_not_matter(oracle):
    t = np.array(UNIT_TRI, np.float32)
    f = t.copy()
    f[[0, 1, 2, 3]] = t[[2, 3, 0, 1]]
    a = oracle.signed_distance(t[:6], (0.5, 0.4))
    b = oracle.signed_distance(f[:6], (0.5, 0.4))
    assert (a > 0) == (b > 0)


def test_opaque_triangle_paints_over_background(oracle):
    img = oracle.render_batch(np.array([[UNIT_TRI]], np.float32), 64, 64, 0.002)[0]
    inside = img[25, 32]
    assert inside[0] > 0.99 and inside[1] < 0.01
    assert np.array_equal(img[63, 0], [0.0, 0.0, 0.0])


def test_offscreen_triangle_is_culled(oracle):
    p = np.array([[tri([[5.0, 5.0], [6.0, 5.0], [5.5, 6.0]], [1, 1, 1], 1.0)]])
    img = oracle.render_batch(p, 32, 32, 0.01, background=(0.1, 0.1, 0.1))
    assert np.all(np.abs(img - 0.1) < 1e-6)
    assert oracle.pixel_bounds(p[0, 0], 32, 32, 0.01) is None


def test_pixel_bounds_pad_and_clamp(oracle):
    # raster.rs:161-167: floor((lo - 6 sigma) * n) clamped at 0, ceil(hi...) + 1 clamped at n.
    t = np.array(UNIT_TRI, np.float32)
    assert oracle.pixel_bounds(t, 64, 64, 0.002) == (12, 12, 53, 53)
    assert oracle.pixel_bounds(t, 64, 64, 0.0) == (12, 12, 53, 53)
    big = tri([[-1.0, -1.0], [2.0, -1.0], [0.5, 2.0]], [1, 1, 1], 1.0)
    assert oracle.pixel_bounds(big, 16, 8, 0.01) == (0, 0, 16, 8)
    nan = big.copy()
    nan[0] = np.nan
    assert oracle.pixel_bounds(nan, 16, 8, 0.01) is None


# --- grad.rs:348-494 --------------------------------------------------------


def test_tape_render_matches_plain_render(oracle):
    scene, _, bg = scene_pair()
    plain = oracle.render_batch(scene[None], 48, 48, 0.02, bg)
    _, _, taped = oracle.backward_batch(scene[None], plain, 0.02, bg, want_images=True)
    assert np.array_equal(plain, taped)


def test_analytic_gradient_matches_finite_differences(oracle):
    scene, tgt, bg = scene_pair()
    target = oracle.render_batch(tgt[None], 48, 48, 0.03, bg)
    loss, analytic = oracle.backward_batch(scene[None], target, 0.03, bg)
    fd_loss, numeric = oracle.finite_difference(scene, 48, 48, 0.03, target[0], bg, 1e-3)
    assert abs(loss[0] - fd_loss) < 1e-6
    norm = max(np.sqrt(np.sum(numeric.astype(np.float64) ** 2)), 1e-8)
    err = np.abs(analytic[0] - numeric) / norm
    assert err.max() < 0.02, err.max()


def test_color_gradient_is_exact_for_a_single_triangle(oracle):
    t = tri([[0.2, 0.25], [0.85, 0.35], [0.5, 0.8]], [0.6, 0.4, 0.2], 1.0)
    tt = t.copy()
    tt[6:9] = [0.1, 0.9, 0.5]
    target = oracle.render_batch(tt[None, None], 32, 32, 0.02)
    _, analytic = oracle.backward_batch(t[None, None], target, 0.02)
    _, numeric = oracle.finite_difference(t[None], 32, 32, 0.02, target[0], eps=1e-3)
    for ch in range(3):
        a, n = analytic[0, 0, 6 + ch], numeric[0, 6 + ch]
        assert abs(a - n) / max(abs(n), 1e-6) < 0.01


def test_batch_gradients_match_sequential_ones(oracle):
    scene, tgt, bg = scene_pair()
    target = oracle.render_batch(tgt[None], 48, 48, 0.02, bg)
    batched = oracle.backward_batch(np.repeat(scene[None], 4, 0), np.repeat(target, 4, 0), 0.02, bg)
    single = oracle.backward_batch(scene[None], target, 0.02, bg, threads=1)
    for b in range(4):
        assert batched[0][b] == single[0][0]
        assert np.array_equal(batched[1][b], single[1][0])


def test_batch_render_matches_sequential_render(oracle):
    scene, _, bg = scene_pair()
    imgs = oracle.render_batch(np.repeat(scene[None], 3, 0), 48, 48, 0.01, bg)
    one = oracle.render_batch(scene[None], 48, 48, 0.01, bg)[0]
    for b in range(3):
        assert np.array_equal(imgs[b], one)


def test_batch_preserves_input_order(oracle):
    params, targets, bgs = [], [], []
    for i in range(6):
        shade = i / 6.0
        params.append(tri([[0.2, 0.2], [0.8, 0.3], [0.5, 0.8]], [1, 0, 0], 0.5)[None])
        bgs.append([shade] * 3)
        targets.append(np.full((16, 16, 3), [1.0 - shade, 0.5, 0.5], np.float32))
    params, targets, bgs = np.stack(params), np.stack(targets), np.array(bgs, np.float32)
    losses, _ = oracle.backward_batch(params, targets, 0.02, bgs)
    for i in range(6):
        l1, _ = oracle.backward_batch(params[i:i + 1], targets[i:i + 1], 0.02, bgs[i])
        assert losses[i] == l1[0]


def test_zero_loss_gives_zero_gradient(oracle):
    scene, _, bg = scene_pair()
    rendered = oracle.render_batch(scene[None], 48, 48, 0.02, bg)
    loss, grads = oracle.backward_batch(scene[None], rendered, 0.02, bg)
    assert loss[0] == 0.0
    assert np.all(grads == 0.0)


def test_clamped_alpha_receives_no_gradient(oracle):
    p = tri([[0.2, 0.2], [0.8, 0.3], [0.5, 0.8]], [1, 0, 0], 1.0)[None, None]
    target = np.zeros((1, 32, 32, 3), np.float32)
    target[..., 2] = 1.0
    _, grads = oracle.backward_batch(p, target, 0.02)
    assert grads[0, 0, 9] == 0.0


def test_culled_triangle_contributes_no_gradient(oracle):
    p = tri([[5.0, 5.0], [6.0, 5.0], [5.5, 6.0]], [1, 1, 1], 1.0)[None, None]
    target = np.full((1, 32, 32, 3), 0.9, np.float32)
    _, grads = oracle.backward_batch(p, target, 0.02, (0.2, 0.2, 0.2))
    assert np.all(grads == 0.0)


# --- optim.rs:63-98 ---------------------------------------------------------


def test_adam_descends_a_quadratic(oracle):
    adam = oracle.Adam(1)
    p = np.zeros(1, np.float32)
    for _ in range(500):
        adam.step(p, 2.0 * (p - 3.0), [0.1])
    assert abs(p[0] - 3.0) < 1e-2
    assert adam.steps_taken == 500


def test_adam_zero_gradient_leaves_params_untouched(oracle):
    adam = oracle.Adam(3)
    p = np.array([1.0, -2.0, 0.5], np.float32)
    before = p.copy()
    adam.step(p, [0.0] * 3, [0.1] * 3)
    assert np.array_equal(p, before)


def test_adam_per_parameter_rates_are_respected(oracle):
    adam = oracle.Adam(2)
    p = np.zeros(2, np.float32)
    adam.step(p, [1.0, 1.0], [0.5, 0.01])
    assert abs(p[0]) > abs(p[1]) * 10.0


def test_powi_is_square_and_multiply(oracle):
    for base in (0.9, 0.999, 1.5):
        for t in range(1, 40):
            exact = float(np.float32(base)) ** t
            assert abs(oracle.powi(base, t) - exact) <= 1e-6 * exact
    assert oracle.powi(0.5, -2) == 4.0


# --- fit.rs:442-635 and tests/integration.rs ---------------------------------


def fit_init(oracle, target, tris, seed):
    from diffrast.scenes import seed_scene_geometry

    p = seed_scene_geometry(tris, seed)
    bg = oracle.seed_colors(target, p)
    return p, bg


def test_sigma_anneals_from_start_to_end(oracle):
    assert abs(oracle.sigma_at(0.02, 0.0015, 100, 0) - 0.02) < 1e-9
    assert abs(oracle.sigma_at(0.02, 0.0015, 100, 99) - 0.0015) < 1e-9
    for i in range(1, 100):
        assert oracle.sigma_at(0.02, 0.0015, 100, i) < oracle.sigma_at(0.02, 0.0015, 100, i - 1)


def test_single_iteration_config_uses_final_sigma(oracle):
    assert oracle.sigma_at(0.02, 0.0015, 1, 0) == np.float32(0.0015)


def test_projection_keeps_parameters_in_range(oracle):
    p = np.array([-5.0, 5.0, 0.5, 0.5, 0.5, 0.5, -1.0, 2.0, 0.5, 1.7], np.float32)
    oracle.project(p)
    assert list(p[0:2]) == [-0.25, 1.25]
    assert list(p[6:9]) == [0.0, 1.0, 0.5]
    assert p[9] == np.float32(0.999)


def test_projection_replaces_non_finite_parameters(oracle):
    p = np.array([np.nan, np.inf, 0.5, 0.5, 0.5, 0.5, np.nan, 0.2, 0.3, np.nan], np.float32)
    oracle.project(p)
    assert np.all(np.isfinite(p))


def _target(oracle, size):
    s, bg = fit_target_scene()
    return oracle.render_batch(s[None], size, size, 0.002, bg)[0]


def test_loss_decreases_on_a_synthetic_target(oracle):
    target = _target(oracle, 48)
    p, bg = fit_init(oracle, target, 16, 7)
    r = oracle.fit(target, p, bg, oracle.FitConfig(iters=200))
    first = r.losses[0]
    assert r.best_loss < first * 0.5
    assert np.isfinite(r.best_loss)
    assert first / r.best_loss > 2.0


def test_fitting_is_deterministic_for_a_fixed_seed(oracle):
    target = _target(oracle, 32)
    p, bg = fit_init(oracle, target, 8, 42)
    a = oracle.fit(target, p, bg, oracle.FitConfig(iters=30))
    b = oracle.fit(target, p, bg, oracle.FitConfig(iters=30))
    assert np.array_equal(a.losses, b.losses)
    assert np.array_equal(a.best_params, b.best_params)


def test_best_scene_is_returned_not_the_last(oracle):
    target = _target(oracle, 40)
    p, bg = fit_init(oracle, target, 12, 3)
    r = oracle.fit(target, p, bg, oracle.FitConfig(iters=150))
    assert r.best_loss <= r.losses[-1]
    assert r.best_loss == r.losses[r.best_iter]


def test_patience_stops_a_stalled_fit_early(oracle):
    target = np.full((24, 24, 3), 0.4, np.float32)
    p, bg = fit_init(oracle, target, 4, 0)
    r = oracle.fit(target, p, bg, oracle.FitConfig(iters=1000, patience=5))
    assert r.stop_reason == oracle.STOP_CONVERGED
    assert len(r.losses) < 1000


def test_invalid_configs_are_rejected(oracle):
    target = np.full((16, 16, 3), 0.5, np.float32)
    p, bg = fit_init(oracle, target, 4, 0)
    cases = [
        (dict(sigma_end=0.0), "NonPositiveSigma"),
        (dict(sigma_start=float("nan")), "NonPositiveSigma"),
        (dict(sigma_start=0.001, sigma_end=0.5), "SigmaNotDecreasing"),
        (dict(lr_pos=-1.0), "NonPositiveLearningRate"),
    ]
    for kw, name in cases:
        with pytest.raises(ValueError, match=name):
            oracle.fit(target, p, bg, oracle.FitConfig(**kw))
    with pytest.raises(ValueError, match="NoTriangles"):
        oracle.fit(target, np.zeros((0, 10), np.float32), bg, oracle.FitConfig())


def test_zero_iterations_is_not_an_error(oracle):
    target = np.full((16, 16, 3), 0.5, np.float32)
    p, bg = fit_init(oracle, target, 4, 0)
    r = oracle.fit(target, p, bg, oracle.FitConfig(iters=0))
    assert len(r.losses) == 0
    assert r.stop_reason == oracle.STOP_COMPLETED


def test_fit_reduces_loss_substantially(oracle):
    s, bg0 = reference_scene()
    target = oracle.render_batch(s[None], 64, 64, 0.002, bg0)[0]
    p, bg = fit_init(oracle, target, 24, 1)
    r = oracle.fit(target, p, bg, oracle.FitConfig(iters=400))
    assert r.losses[0] / r.best_loss > 10.0
    assert r.stop_reason != oracle.STOP_DIVERGED


def test_render_is_deterministic(oracle):
    s, bg = reference_scene()
    a = oracle.render_batch(s[None], 96, 96, 0.004, bg)
    b = oracle.render_batch(s[None], 96, 96, 0.004, bg)
    assert np.array_equal(a, b)


def test_taped_render_matches_plain_render_at_several_sizes(oracle):
    s, bg = reference_scene()
    for (w, h) in [(32, 32), (64, 48), (17, 41)]:
        plain = oracle.render_batch(s[None], h, w, 0.01, bg)
        _, _, taped = oracle.backward_batch(s[None], plain, 0.01, bg, want_images=True)
        assert np.array_equal(plain, taped), (w, h)


def test_gradient_points_downhill(oracle):
    s, bg = reference_scene()
    target = oracle.render_batch(s[None], 48, 48, 0.002, bg)
    scene = s.copy()
    scene[0, 0] += 0.08
    scene[0, 6:9] = 0.3
    loss, grads = oracle.backward_batch(scene[None], target, 0.02, bg)
    g = grads[0].ravel()
    step = np.float32(1e-3) / max(np.float32(np.sqrt(np.sum(g * g))), np.float32(1e-12))
    stepped = (scene.ravel() - step * g).reshape(scene.shape).astype(np.float32)
    new_loss = oracle.mse(oracle.render_batch(stepped[None], 48, 48, 0.02, bg), target)
    assert new_loss < loss[0]


def test_non_square_and_tiny_canvases_are_handled(oracle):
    for (w, h) in [(1, 1), (1, 64), (64, 1), (37, 11)]:
        target = np.full((h, w, 3), [0.4, 0.5, 0.6], np.float32)
        p, bg = fit_init(oracle, target, 4, 0)
        r = oracle.fit(target, p, bg, oracle.FitConfig(iters=10, patience=None))
        assert np.isfinite(r.best_loss), (w, h)


def test_empty_scene_renders_the_background(oracle):
    img = oracle.render_batch(np.zeros((1, 0, 10), np.float32), 16, 16, 0.01, (0.2, 0.4, 0.6))
    assert np.all(img[0] == np.array([0.2, 0.4, 0.6], np.float32))


def test_mse_is_zero_against_itself_and_positive_otherwise(oracle):
    a = np.full((8, 8, 3), [0.25, 0.5, 0.75], np.float32)
    assert oracle.mse(a, a) == 0.0
    b = np.full((8, 8, 3), [0.25, 0.5, 0.70], np.float32)
    assert oracle.mse(a, b) > 0.0


# --- oracle-specific properties -----------------------------------------------


def test_f64_twin_tracks_f32_oracle(oracle):
    scene, tgt, bg = scene_pair()
    target = oracle.render_batch(tgt[None], 48, 48, 0.02, bg)
    l32, g32 = oracle.backward_batch(scene[None], target, 0.02, bg)
    l64, g64 = oracle.backward_batch(scene[None], target, 0.02, bg, f64=True)
    assert abs(l32[0] - l64[0]) <= 1e-6 * abs(l64[0]) + 1e-9
    assert np.max(np.abs(g32 - g64)) <= 1e-4 * np.max(np.abs(g64))


def test_gradient_input_modes_agree(oracle):
    # diffrast-py's target inversion (lib.rs:311-313) vs using dL/dr directly.
    scene, tgt, bg = scene_pair()
    target = oracle.render_batch(tgt[None], 48, 48, 0.02, bg)
    rendered = oracle.render_batch(scene[None], 48, 48, 0.02, bg)
    n = np.float32(48 * 48 * 3)
    g_in = (np.float32(2.0) * (rendered - target) / n).astype(np.float32)
    _, via_target = oracle.backward_batch(scene[None], target, 0.02, bg)
    _, inv = oracle.backward_batch(scene[None], g_in, 0.02, bg, mode=oracle.MODE_INVERT_GRAD)
    _, direct = oracle.backward_batch(scene[None], g_in, 0.02, bg, mode=oracle.MODE_DIRECT_GRAD)
    norm = np.linalg.norm(via_target)
    assert np.max(np.abs(inv - via_target)) / norm < 1e-3
    assert np.max(np.abs(direct - via_target)) / norm < 1e-4


def test_f64_fit_twin_tracks_the_f32_fit(oracle):
    # The f64 twin runs the same fit (sigma schedule and box cull in f32) with
    # f64 parameters, moments and loss: the two start out equal to rounding
    # and drift apart only as f32 rounding accumulates.
    target = np.full((24, 24, 3), 0.4, np.float32)
    target[6:18, 6:18] = (0.9, 0.2, 0.1)
    p = np.zeros((6, 10), np.float32)
    rng = np.random.default_rng(3)
    p[:, :6] = rng.uniform(0.2, 0.8, (6, 6))
    p[:, 6:9] = rng.uniform(0, 1, (6, 3))
    p[:, 9] = 0.5
    cfg = oracle.FitConfig(iters=40, patience=None)
    r32 = oracle.fit(target, p, (0.4, 0.4, 0.4), cfg)
    r64 = oracle.fit(target, p, (0.4, 0.4, 0.4), cfg, f64=True)
    assert r64.losses.dtype == np.float64 and len(r64.losses) == len(r32.losses) == 40
    assert abs(r64.losses[0] - r32.losses[0]) <= 1e-6 * r64.losses[0]
    assert np.all(np.abs(r64.losses - r32.losses) <= 1e-3 * r64.losses)
    assert r64.best_loss < r64.losses[0]
