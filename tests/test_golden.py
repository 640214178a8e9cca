"""Committed golden fixtures (tests/golden/, made by tests/golden/make_golden.py).

CPU: this build's torch helpers reproduce the reference's own Python helpers
(vectors produced by importing the reference's torch_layer.py / model.py), and
the CPU oracle reproduces its committed outputs bit for bit.
GPU: the CUDA path (through the C ABI) matches the committed oracle outputs
within the parity tolerances (images 1e-5 abs + 1e-4 rel, losses 1e-5 rel,
gradients 1e-6 + 1e-3 |ref| per element).
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from conftest import assert_grads_close, assert_images_close

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _helpers():
    return np.load(os.path.join(GOLDEN, "reference_torch_helpers.npz"))


def _cases():
    z = np.load(os.path.join(GOLDEN, "oracle_cases.npz"))
    names = sorted({k.split("/")[0] for k in z.files})
    return z, names


CASE_NAMES = _cases()[1]


def test_random_params_matches_the_reference():
    from diffrast import torch_layer

    z = _helpers()
    for seed, (b, t) in ((0, (2, 5)), (7, (3, 16)), (123, (1, 64))):
        g = torch.Generator().manual_seed(seed)
        got = torch_layer.random_params(b, t, generator=g).numpy()
        np.testing.assert_array_equal(got, z[f"random_params_s{seed}"])


def test_clamp_params_matches_the_reference():
    from diffrast import torch_layer

    z = _helpers()
    got = torch_layer.clamp_params(torch.from_numpy(z["clamp_in"])).numpy()
    np.testing.assert_array_equal(got, z["clamp_out"])


def test_activate_matches_the_reference():
    from diffrast import torch_layer

    z = _helpers()
    raw = torch.from_numpy(z["activate_in"])
    for vr in (0.15, 0.0, 0.3):
        got = torch_layer.activate(raw, vertex_range=vr).numpy()
        np.testing.assert_array_equal(got, z[f"activate_out_vr{vr}"])


def test_psnr_matches_the_reference():
    from diffrast import torch_layer

    z = _helpers()
    a, b = torch.from_numpy(z["psnr_a"]), torch.from_numpy(z["psnr_b"])
    assert np.float32(torch_layer.psnr(a, b).item()) == z["psnr_ab"]
    assert np.float32(torch_layer.psnr(a, a).item()) == z["psnr_aa"]


@pytest.mark.parametrize("name", CASE_NAMES)
def test_oracle_reproduces_golden(oracle, name):
    z, _ = _cases()
    p, tgt = z[f"{name}/params"], z[f"{name}/target"]
    sigma, bg = float(z[f"{name}/sigma"]), z[f"{name}/background"]
    H, W = tgt.shape[1], tgt.shape[2]
    img = oracle.render_batch(p, H, W, sigma, bg)
    np.testing.assert_array_equal(img, z[f"{name}/image"])
    losses, grads = oracle.backward_batch(p, tgt, sigma, bg)
    np.testing.assert_array_equal(losses, z[f"{name}/losses"])
    np.testing.assert_array_equal(grads, z[f"{name}/grads"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASE_NAMES)
def test_cuda_matches_golden(name):
    from diffrast import _native

    z, _ = _cases()
    p = torch.from_numpy(z[f"{name}/params"]).cuda()
    tgt = torch.from_numpy(z[f"{name}/target"]).cuda()
    sigma, bg = float(z[f"{name}/sigma"]), z[f"{name}/background"]
    H, W = tgt.shape[1], tgt.shape[2]
    img = _native.render(p, H, W, sigma, bg)
    assert_images_close(img.cpu().numpy(), z[f"{name}/image"], f"{name} image")
    losses, grads, img2 = _native.loss_backward(p, tgt, sigma, bg, want_image=True)
    if not np.isnan(z[f"{name}/params"][..., 9]).any():
        # The backward's tape drops NaN-alpha triangles, which render() paints
        # (grad.rs:62 vs raster.rs:49); elsewhere both images agree.
        assert_images_close(img2.cpu().numpy(), z[f"{name}/image"], f"{name} loss-pass image")
    ref_l = z[f"{name}/losses"]
    np.testing.assert_allclose(losses.cpu().numpy(), ref_l, rtol=1e-5, atol=1e-12)
    assert_grads_close(grads.cpu().numpy(), z[f"{name}/grads"], f"{name} grads")


def test_bbox_pair_count_matches_the_oracle_boxes(oracle):
    # The roofline's unit of work, counted on the host with numpy, against the
    # oracle's pixel_bounds (raster.rs:144-168) triangle by triangle.
    from diffrast.scenes import bbox_pairs, config5_params, uniform_scenes

    rng = np.random.default_rng(12)
    p = np.concatenate([uniform_scenes(3, 40, 9), config5_params(2, 40, 5300)], axis=0)
    p[0, :5, :6] = rng.uniform(-0.5, 1.5, (5, 6))  # partly or wholly off the canvas
    p[1, 3, 0] = np.nan
    p[1, 4, 9] = 0.0
    for (w, h, sigma) in ((256, 256, 0.0015), (37, 45, 0.02), (1, 1, 0.0)):
        want = 0
        for tri in p.reshape(-1, 10):
            if not (tri[9] > 0):
                continue
            bb = oracle.pixel_bounds(tri, w, h, sigma)
            if bb:
                want += (bb[2] - bb[0]) * (bb[3] - bb[1])
        assert bbox_pairs(p, w, h, sigma) == want, (w, h, sigma)
