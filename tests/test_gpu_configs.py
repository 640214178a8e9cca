"""Parity at the benchmark configurations themselves, full size.

Each test runs the CUDA path on exactly the inputs a benchmark times (the same
seeds, batch, triangle count, canvas and sigma) and compares it with the CPU
oracle, per element, at the north star's tolerances:
- images |d| <= 1e-5 + 1e-4 |ref|;
- losses relative 1e-5;
- gradients |d| <= 1e-6 + 1e-3 |ref|, plus the reference's own metric
  max|d| / ||ref|| < 1e-3 per scene (diffrast-gpu/src/lib.rs:1252-1254).

Config 1 (the 800-iteration fit) is judged against the spread between the
f32 oracle and its f64 twin: a fit amplifies rounding differences, and that
spread is the size of the difference f32 rounding alone makes.

Set DR_REPORT_DIR to write the measured errors of each case as JSON there.
"""

from __future__ import annotations

import json
import os
import threading

import numpy as np
import pytest

from conftest import assert_grads_close, assert_images_close, rel_norm_error

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


def report(name, **values):
    d = os.environ.get("DR_REPORT_DIR")
    if not d:
        return
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, f"parity_{name}.json"), "w") as f:
        json.dump(values, f, indent=1, default=float)


def max_excess(got, ref):
    """Largest |d| / (1e-6 + 1e-3 |ref|) over the elements (<= 1 passes)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    ok = ~np.isnan(ref)
    return float(np.max(np.abs(got[ok] - ref[ok]) / (1e-6 + 1e-3 * np.abs(ref[ok])), initial=0.0))


def full_parity(native, oracle, params, target, sigma, bg=(0.0, 0.0, 0.0), name="case"):
    """Render, fused loss + backward (image, loss, grads) and the upstream-
    gradient backward of one batch, each against the oracle."""
    B = params.shape[0]
    H, W = target.shape[1], target.shape[2]
    img = host(native.render(cuda(params), H, W, sigma, bg))
    ref_img = oracle.render_batch(params, H, W, sigma, bg)
    assert_images_close(img, ref_img, f"{name} render")

    losses, grads, img2 = native.loss_backward(cuda(params), cuda(target), sigma, bg,
                                               want_image=True)
    losses, grads, img2 = host(losses), host(grads), host(img2)
    ref_l, ref_g, ref_img2 = oracle.backward_batch(params, target, sigma, bg, want_images=True)
    assert_images_close(img2, ref_img2, f"{name} fused render")
    np.testing.assert_allclose(losses, ref_l, rtol=1e-5, atol=1e-9)
    assert_grads_close(grads, ref_g, f"{name} loss grads")
    rel = [rel_norm_error(grads[b], ref_g[b]) for b in range(B)]
    assert max(rel) < 1e-3

    g_in = np.random.default_rng(7).normal(0, 1e-4, size=target.shape).astype(np.float32)
    gg = host(native.grad_backward(cuda(params), cuda(g_in), sigma, bg))
    _, ref_gg = oracle.backward_batch(params, g_in, sigma, bg, mode=oracle.MODE_DIRECT_GRAD)
    assert_grads_close(gg, ref_gg, f"{name} grad-input grads")
    report(name, image_max_abs=float(np.nanmax(np.abs(img2 - ref_img2))),
           loss_max_rel=float(np.max(np.abs(losses - ref_l) / np.abs(ref_l))),
           grad_max_excess=max_excess(grads, ref_g), grad_rel_norm_max=max(rel),
           grad_input_max_excess=max_excess(gg, ref_gg),
           path=native.query_path(B, params.shape[1], H, W))
    return img2, grads


def test_headline_cell_through_the_region_kernel(native, oracle):
    # The cell bench.py times: config 2, B=32, T=128, 256^2, sigma 0.0015,
    # params seed 2005, target scenes seed 3005 rendered at the same sigma.
    from diffrast.scenes import config2_params

    p, tp = config2_params(32, 128, 5)
    assert native.query_path(32, 128, 256, 256) == native.PATH_REGION
    target = oracle.render_batch(tp, 256, 256, 0.0015)
    full_parity(native, oracle, p, target, 0.0015, name="headline")


@pytest.mark.parametrize("T", [32, 128, 512])
@pytest.mark.parametrize("size", [64, 128, 256])
def test_config2_cells_full_batch(native, oracle, T, size):
    from diffrast.scenes import config2_params

    cell = [32, 128, 512].index(T) * 3 + [64, 128, 256].index(size)
    p, tp = config2_params(32, T, cell)
    if T == 512:  # lists gathered from the tile masks
        assert native.query_path(32, T, size, size) == native.PATH_TILE_GATHER
    target = oracle.render_batch(tp, size, size, 0.0015)
    full_parity(native, oracle, p, target, 0.0015, name=f"config2_T{T}_{size}")


@pytest.mark.parametrize("T", [128, 512])
def test_config2_wide_band_cells(native, oracle, T):
    # Config 2's second sigma (0.01): bands wide against an 8x4 block, where
    # the classification prunes candidate edges with its corner bounds.
    from diffrast.scenes import config2_params

    cell = [32, 128, 512].index(T) * 3 + 2
    p, tp = config2_params(32, T, cell)
    target = oracle.render_batch(tp, 256, 256, 0.01)
    full_parity(native, oracle, p, target, 0.01, name=f"config2_T{T}_256_s0.01")


def test_config3_torch_op_full_batch(native, oracle):
    # Config 3 exactly as the bench times it: activate(raw) params for 256
    # scenes of 64 triangles, targets rendered from random_params, then
    # rasterize -> F.mse_loss -> backward (the forward keeps the pixel tape).
    import torch.nn.functional as F

    from diffrast import torch_layer

    raw = torch.randn(256, 64, 10, generator=torch.Generator().manual_seed(2))
    params = torch_layer.activate(raw)
    tparams = torch_layer.random_params(256, 64, generator=torch.Generator().manual_seed(3))
    targets = torch_layer.rasterize(tparams.cuda(), 128, 128, 0.0015).detach()
    q = params.cuda().requires_grad_(True)
    img = torch_layer.rasterize(q, 128, 128, 0.0015)
    loss = F.mse_loss(img, targets)
    loss.backward()
    p_np = params.numpy()
    t_hwc = targets.permute(0, 2, 3, 1).contiguous().cpu().numpy()
    ref_l, ref_g, ref_img = oracle.backward_batch(p_np, t_hwc, 0.0015, want_images=True)
    assert_images_close(host(img).transpose(0, 2, 3, 1), ref_img, "config 3 render")
    np.testing.assert_allclose(float(loss.detach()), float(np.mean(ref_l)), rtol=1e-5)
    # F.mse_loss averages over the whole batch: the per-scene gradients / B.
    assert_grads_close(host(q.grad), ref_g / 256, "config 3 grads")
    report("config3", image_max_abs=float(np.nanmax(np.abs(host(img).transpose(0, 2, 3, 1) -
                                                           ref_img))),
           grad_max_excess=max_excess(host(q.grad), ref_g / 256),
           path=native.query_path(256, 64, 128, 128))


def test_config4_full_scene(native, oracle):
    # Config 4: one 1024^2 scene of 4096 small triangles (gathered tile lists).
    from diffrast.scenes import config4_params

    p = config4_params(4096, 4000)
    assert native.query_path(1, 4096, 1024, 1024) == native.PATH_TILE_GATHER
    target = oracle.render_batch(config4_params(4096, 4001), 1024, 1024, 0.0015)
    full_parity(native, oracle, p, target, 0.0015, name="config4")


@pytest.mark.parametrize("sigma", [0.00015, 0.0015, 0.015])
def test_config5_full_batch(native, oracle, sigma):
    # All 16 seeded stress scenes (seeds 5000..5015): heavy overlap, 5 %
    # degenerate triangles, opacity exactly 0 and 1.
    from diffrast.scenes import config5_params

    p = config5_params(16, 2048, 5000)
    assert native.query_path(16, 2048, 512, 512) == native.PATH_TILE_GATHER
    target = oracle.render_batch(config5_params(16, 2048, 5100), 512, 512, sigma)
    img, grads = full_parity(native, oracle, p, target, sigma, name=f"config5_{sigma}")
    ref_img = oracle.render_batch(p, 512, 512, sigma)
    assert np.count_nonzero(~np.isfinite(img)) == np.count_nonzero(~np.isfinite(ref_img)) == 0
    assert np.isfinite(grads).all()
    assert np.all(grads[p[..., 9] == 0.0] == 0.0)        # alpha 0: no gradient
    assert np.all(grads[p[..., 9] == 1.0][:, 9] == 0.0)  # alpha 1: alpha pinned


def test_config1_full_fit_within_the_f32_noise_floor(native, oracle):
    # Config 1: 150 triangles (seed 0) rendered at 176^2 by the forward, fit
    # from a seed-1 init for 800 iterations with FitConfig defaults otherwise.
    from diffrast.scenes import config1_target_scene, seed_scene_geometry

    target = oracle.render_batch(config1_target_scene(150, 0), 176, 176, 0.0015)[0]
    p = seed_scene_geometry(150, 1)
    bg = oracle.seed_colors(target, p)
    cfg = oracle.FitConfig(iters=800)
    out = {}

    def run(key, f64):
        out[key] = oracle.fit(target, p, bg, cfg, f64=f64)

    threads = [threading.Thread(target=run, args=(k, f)) for k, f in (("f32", False),
                                                                         ("f64", True))]
    for t in threads:
        t.start()
    got = native.fit(torch.from_numpy(target).cuda(), torch.from_numpy(p).cuda(),
                     [float(v) for v in bg], iters=800)
    for t in threads:
        t.join()
    r32, r64 = out["f32"], out["f64"]
    lg = host(got["losses"]).astype(np.float64)
    l32, l64 = r32.losses.astype(np.float64), r64.losses
    assert len(lg) == len(l32) == len(l64) == 800
    assert got["stop_reason"] == r32.stop_reason

    # The noise floor at iteration i: the largest f32-vs-f64 relative spread
    # seen up to i (a running envelope), floored at a few f32 ulps.
    spread = np.maximum.accumulate(np.abs(l32 - l64) / l64)
    floor = np.maximum(spread, 4 * 2.0 ** -24)
    dev = np.abs(lg - l32) / l32
    ratio = dev / floor
    first = int(np.argmax(dev > 1e-4)) if (dev > 1e-4).any() else 800
    report("config1_fit", first_divergence_1e4=first, max_ratio_to_floor=float(ratio.max()),
           dev_at=[float(dev[i]) for i in (0, 10, 50, 100, 200, 400, 799)],
           spread_at=[float(spread[i]) for i in (0, 10, 50, 100, 200, 400, 799)],
           best_loss=[float(got["best_loss"]), float(r32.best_loss), float(r64.best_loss)],
           final_param_dist=[float(np.linalg.norm(host(got["final_params"]) - r32.final_params)),
                             float(np.linalg.norm(r32.final_params - r64.final_params))])
    # The GPU's loss curve stays within a small multiple of the f32 noise floor
    # over the whole fit.
    assert ratio.max() <= 16.0, (int(np.argmax(ratio)), float(ratio.max()))
    # Best loss and final parameters differ from the f32 oracle by no more
    # than f32 rounding makes the oracle differ from its f64 twin (with the same
    # margin).
    assert abs(got["best_loss"] - r32.best_loss) <= 16 * max(
        abs(r32.best_loss - r64.best_loss), 4 * 2.0 ** -24 * r32.best_loss)
    d_gpu = np.linalg.norm(host(got["final_params"]) - r32.final_params)
    d_f64 = np.linalg.norm(r32.final_params - r64.final_params)
    assert d_gpu <= 4 * d_f64 + 1e-6
    d_best_gpu = np.linalg.norm(host(got["best_params"]) - r32.best_params)
    d_best_f64 = np.linalg.norm(r32.best_params - r64.best_params)
    assert d_best_gpu <= 4 * d_best_f64 + 1e-6
