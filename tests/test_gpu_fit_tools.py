"""The fit loop's callers on the GPU: the step-wise Fitter against the graph
fit (dr_fit), checkpoint/resume, the refine loop of evaluate.py, and the fit
CLI end to end (fit.rs, python/evaluate.py:79-132, bin/fit.rs)."""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def small_target():
    from diffrast import _native
    from diffrast.scenes import config1_target_scene

    p = torch.from_numpy(config1_target_scene(40, 0)).cuda()
    return _native.render(p, 48, 56, 0.0015)[0].cpu().numpy()


def test_stepwise_fitter_matches_the_graph_fit():
    from diffrast.fit import FitConfig, Fitter, fit

    tgt = small_target()
    cfg = FitConfig(triangles=24, iters=60, seed=5)
    graph = fit(tgt, cfg)
    f = Fitter(tgt, cfg)
    while f.step() is not None:
        pass
    step = f.report()
    assert step.stop_reason == graph.stop_reason
    assert len(step.losses) == len(graph.losses) == 60
    # Same kernels; gradients are f32 atomic sums whose order varies run to
    # run, and a fit amplifies those ulp differences step by step (the f32
    # oracle and its f64 twin drift apart the same way). The first steps agree
    # tightly, the rest within half a percent.
    np.testing.assert_allclose(step.losses[:10], graph.losses[:10], rtol=1e-5)
    np.testing.assert_allclose(step.losses, graph.losses, rtol=5e-3)
    assert step.best_loss < step.losses[0]


def test_checkpoint_and_resume_continue_exactly(tmp_path):
    from diffrast.fit import FitConfig, Fitter

    tgt = small_target()
    cfg = FitConfig(triangles=16, iters=40, seed=2, patience=None)
    a = Fitter(tgt, cfg)
    for _ in range(15):
        a.step()
    a.save(tmp_path / "ck.npz")
    b = Fitter.from_state(tgt, str(tmp_path / "ck.npz"))
    assert b.iter == 15 and b.losses == a.losses
    assert torch.equal(a.params, b.params) and torch.equal(a.m, b.m) and torch.equal(a.v, b.v)
    while a.step() is not None:
        pass
    while b.step() is not None:
        pass
    ra, rb = a.report(), b.report()
    np.testing.assert_allclose(ra.losses, rb.losses, rtol=1e-5)
    assert ra.best_iter == rb.best_iter


def test_diverged_fit_stops_and_keeps_the_best():
    from diffrast.fit import FitConfig, Fitter, StopReason

    tgt = small_target()
    tgt[0, 0, 0] = np.nan  # a NaN target makes the first loss NaN
    f = Fitter(tgt, FitConfig(triangles=8, iters=10))
    assert f.step() is None
    assert f.report().stop_reason == StopReason.DIVERGED


def test_refine_matches_the_reference_torch_loop():
    # evaluate.py:79-132 with torch's Adam over fused_loss, restated here as
    # the comparison; refine() uses the fused device Adam.
    from diffrast import torch_layer as tl
    from diffrast.refine import mse_to_psnr, refine

    g = torch.Generator().manual_seed(0)
    targets = tl.rasterize(tl.random_params(3, 12, generator=g).cuda(), 32, 32,
                           sigma=0.004).detach()
    start = tl.random_params(3, 12, generator=torch.Generator().manual_seed(1)).cuda()
    p_ref = start.clone()
    opt = torch.optim.Adam([p_ref], lr=0.02)
    hwc = targets.permute(0, 2, 3, 1).contiguous()
    trace_ref = []
    for _ in range(30):
        losses, grads = tl.fused_loss(p_ref, hwc, sigma=0.004)
        trace_ref.append(mse_to_psnr(losses.mean().item()))
        opt.zero_grad(set_to_none=True)
        p_ref.grad = grads / 3
        opt.step()
        with torch.no_grad():
            p_ref.copy_(tl.clamp_params(p_ref))
    trace_ref.append(mse_to_psnr(tl.fused_loss(p_ref, hwc, sigma=0.004)[0].mean().item()))
    p, trace = refine(start, targets, 30, 0.004)
    assert len(trace) == 31 and trace[0] == pytest.approx(trace_ref[0], abs=1e-9)
    np.testing.assert_allclose(trace, trace_ref, atol=0.05)
    assert trace[-1] > trace[0] + 1.0


def test_fit_cli_writes_the_reference_artefacts(tmp_path):
    from diffrast import fit_cli, formats

    out = tmp_path / "run"
    rc = fit_cli.run(["--tris", "16", "--iters", "30", "--size", "40", "--export", "64",
                      "--save-every", "10", "--out", str(out), "--quiet",
                      "--checkpoint", str(tmp_path / "ck.npz")])
    assert rc == 0
    for name in ("target.png", "fit.png", "loss.csv", "scene.json"):
        assert (out / name).exists(), name
    assert formats.read_png(out / "target.png").shape == (40, 40, 3)
    assert formats.read_png(out / "fit.png").shape == (64, 64, 3)
    assert sorted(os.listdir(out / "frames")) == [f"frame_0000{i}.png" for i in range(3)]
    scene = json.loads((out / "scene.json").read_text())
    assert scene["version"] == 1 and len(scene["triangles"]) == 16
    rows = (out / "loss.csv").read_text().splitlines()
    assert rows[0] == "iter,loss" and len(rows) == 31
    # Resume the saved fit for 20 more iterations.
    out2 = tmp_path / "run2"
    rc = fit_cli.run(["--iters", "50", "--size", "40", "--export", "64", "--out", str(out2),
                      "--quiet", "--resume", str(tmp_path / "ck.npz")])
    assert rc == 0
    rows2 = (out2 / "loss.csv").read_text().splitlines()
    assert rows2[:31] == rows


def test_fit_cli_graph_path_and_png_target(tmp_path):
    from diffrast import fit_cli, formats

    tgt = tmp_path / "t.png"
    formats.write_png(tgt, small_target())
    rc = fit_cli.run([str(tgt), "--tris", "16", "--iters", "20", "--size", "28", "--export",
                      "56", "--out", str(tmp_path / "o"), "--quiet"])
    assert rc == 0
    assert formats.read_png(tmp_path / "o" / "target.png").shape == (24, 28, 3)
    assert formats.read_png(tmp_path / "o" / "fit.png").shape == (48, 56, 3)
