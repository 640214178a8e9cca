"""``python bench_kernels.py``: the path's memory-bound kernels alone.

Prints one JSON line per kernel with its algorithmic bytes, CUDA-event time
and achieved GB/s against the measured HBM peak. All sizes are far above the
126 MB L2:
- ``dr_setup_kernel``: 40 B of parameters read and one 160-byte record written
  per triangle. It is timed inside ``dr_render`` of 1x1 images, whose raster
  part is tiny; use ncu's per-kernel time for the kernel alone.
- ``dr_mse_kernel`` (``dr_mse_loss``): two f32 images read.
- ``dr_adam_kernel`` (``dr_adam_step``): parameters, moments and gradient read
  (16 B), parameters and moments written (12 B), per parameter.

The first call of each is the measured size, so an ncu capture of the first
launch of each kernel (``-c 3``) sees the same work.

``--fit-iters N`` instead runs the config 1 fit (150 triangles, 176x176) for
N iterations through ``dr_fit`` (one CUDA graph) twice, and prints the second
run's time per iteration: a short driver for the fit graph's launch list.

``--config C`` instead runs ``--steps`` loss + backward calls of one benchmark
configuration whose scenes take the tile kernel's gathered lists (C = 4: one
1024^2 scene of 4096 triangles; 5: 16 scenes of 2048 triangles at 512^2;
2-512: 32 scenes of 512 triangles at 256^2; 2-128: the headline cell, 128
triangles at 256^2, whose first ``--batch`` scenes (default 32) are one
rank's share under strong scaling; all at sigma 0.0015), after one render of
the target: a short driver for an ncu capture of the raster kernel (skip the
first raster launch, the target's render).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "differentiable-rasterizer_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

from diffrast import _native  # noqa: E402

REC_BYTES = 160


def _peak_gbs() -> tuple[float, str]:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s"


def _time(fn, reps: int) -> float:
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--fit-iters", type=int, default=0)
    ap.add_argument("--config", choices=("4", "5", "2-512", "2-128"))
    ap.add_argument("--batch", type=int, default=32, help="scenes of config 2-128")
    ap.add_argument("--forward", action="store_true",
                    help="with --config: time the forward alone (dr_render, BCHW)")
    ap.add_argument("--steps", type=int, default=3)
    args = ap.parse_args(argv)
    if args.fit_iters > 0:
        fit_graph(args.fit_iters)
        return
    if args.config:
        config_steps(args.config, args.steps, args.batch, args.forward)
        return
    peak, src = _peak_gbs()
    g = torch.Generator(device="cuda").manual_seed(0)

    def line(name, nbytes, ms, work):
        gbs = nbytes / (ms * 1e-3) / 1e9
        print(json.dumps({"kernel": name, "work": work, "bytes": nbytes, "ms": ms,
                          "gb_s": gbs, "peak_gb_s": peak, "frac": gbs / peak,
                          "peak_source": src}), flush=True)

    B, T = 256, 4096
    params = torch.rand(B, T, 10, device="cuda", generator=g)
    ms = _time(lambda: _native.render(params, 1, 1, 0.0015), args.reps)
    line("dr_setup_kernel (+ 1x1 raster)", B * T * (40 + REC_BYTES), ms,
         f"{B * T} triangles")

    Bm, n = 64, 512 * 512 * 3
    a = torch.rand(Bm, 512, 512, 3, device="cuda", generator=g)
    b = torch.rand(Bm, 512, 512, 3, device="cuda", generator=g)
    ms = _time(lambda: _native.mse_loss(a, b), args.reps)
    line("dr_mse_kernel", 2 * 4 * Bm * n, ms, f"{Bm} images of 512x512x3")

    npar = 16 * 1024 * 1024
    p = torch.rand(npar, device="cuda", generator=g)
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    gr = torch.randn(npar, device="cuda", generator=g) * 1e-3
    step = [0]

    def adam():
        step[0] += 1
        _native.adam_step(p, m, v, gr, step[0])

    ms = _time(adam, args.reps)
    line("dr_adam_kernel", 28 * npar, ms, f"{npar} parameters")


def config_steps(config: str, steps: int, batch: int = 32, forward: bool = False) -> None:
    from diffrast import scenes as S

    if config == "4":
        p, tp, size = S.config4_params(4096, 4000), S.config4_params(4096, 4001), 1024
    elif config == "5":
        p, tp, size = S.config5_params(16, 2048, 5000), S.config5_params(16, 2048, 5100), 512
    elif config == "2-128":
        (p, tp), size = S.config2_params(32, 128, 5), 256
        p, tp = p[:batch], tp[:batch]
    else:
        (p, tp), size = S.config2_params(32, 512, 8), 256
    P = torch.from_numpy(p).cuda()
    target = _native.render(torch.from_numpy(tp).cuda(), size, size, 0.0015)
    path = _native.query_path(P.shape[0], P.shape[1], size, size)
    if forward:
        call = lambda: _native.render(P, size, size, 0.0015, layout=_native.LAYOUT_BCHW)  # noqa: E731
    else:
        call = lambda: _native.loss_backward(P, target, 0.0015)  # noqa: E731
    ms = [_time(call, 1) for _ in range(steps)]
    print(json.dumps({"config": config, "B": P.shape[0], "T": P.shape[1], "size": size,
                      "path": path, "forward": forward, "ms_per_call": ms}), flush=True)


def fit_graph(iters: int) -> None:
    from diffrast.fit import mean_color, seed_colors
    from diffrast.scenes import config1_target_scene, seed_scene_geometry

    target = _native.render(torch.from_numpy(config1_target_scene(150, 0)).cuda(), 176, 176,
                            0.0015)[0].contiguous()
    p = seed_scene_geometry(150, 1)
    seed_colors(target.cpu().numpy(), p)
    bg = [float(x) for x in mean_color(target.cpu().numpy())]
    p_dev = torch.from_numpy(p).cuda()
    _native.fit(target, p_dev, bg, iters=iters, patience=None)  # capture
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    _native.fit(target, p_dev, bg, iters=iters, patience=None)
    e1.record()
    torch.cuda.synchronize()
    print(json.dumps({"fit": "config 1", "iters": iters,
                      "us_per_iter": e0.elapsed_time(e1) * 1e3 / iters}), flush=True)


if __name__ == "__main__":
    main()
