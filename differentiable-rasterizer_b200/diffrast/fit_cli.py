"""``python -m diffrast.fit_cli``: the reference's ``fit`` binary on the GPU
(crates/diffrast/src/bin/fit.rs), same options and outputs, plus checkpoints.

Outputs in ``--out`` (default ``out``): ``target.png``, ``fit.png`` (the best
scene re-rendered with its longest side at ``--export``), ``loss.csv``,
``scene.json``, and ``frames/frame_NNNNN.png`` every ``--save-every``
iterations. ``--checkpoint PATH`` saves the fit state every
``--checkpoint-every`` iterations and at the end; ``--resume PATH`` continues a
saved fit exactly where it stopped.

Without frames or checkpoints the whole loop runs as one CUDA graph
(``dr_fit``); otherwise one device iteration per step (``Fitter``).
"""

from __future__ import annotations

import os
import sys
import time

import numpy as np
import torch

from . import _native, formats
from .fit import ConfigError, FitConfig, Fitter, StopReason, fit

USAGE = """\
fit — reconstruct an image from soft triangles (GPU)

usage: python -m diffrast.fit_cli [target.png] [options]

  --tris N              triangles in the scene        (default 128)
  --iters N             optimizer steps               (default 1500)
  --size N              longest side of the fit       (default 192)
  --out DIR             output directory              (default out)
  --save-every N        write a frame every N iters   (default 0, off)
  --export N            longest side of final render  (default 1024)
  --seed N              RNG seed                      (default 0)
  --patience N          stop after N stalled iters    (default 250, 0 disables)
  --checkpoint PATH     save the fit state here
  --checkpoint-every N  ... every N iters as well as at the end (default 0)
  --resume PATH         continue a fit saved with --checkpoint
  --quiet               suppress per-iteration output
  --help                show this message

With no target image, a synthetic one is generated."""


class UsageError(ValueError):
    pass


def parse_args(argv: list[str]):
    """bin/fit.rs:126-172 plus the checkpoint options. None for --help."""
    if any(a in ("--help", "-h") for a in argv):
        return None
    target = argv[0] if argv and not argv[0].startswith("-") else None
    cfg = FitConfig()
    opts = {"size": 192, "out": "out", "save_every": 0, "export": 1024, "quiet": False,
            "checkpoint": None, "checkpoint_every": 0, "resume": None}
    i = 1 if target is not None else 0

    def num(flag, raw):
        try:
            v = int(raw)
        except ValueError:
            v = -1
        if v < 0 or not raw.isdigit():
            raise UsageError(f"{flag} expects a non-negative integer, got '{raw}'")
        return v

    while i < len(argv):
        flag = argv[i]
        if flag == "--quiet":
            opts["quiet"] = True
            i += 1
            continue
        if flag not in ("--tris", "--iters", "--size", "--seed", "--export", "--save-every",
                        "--patience", "--out", "--checkpoint", "--checkpoint-every", "--resume"):
            raise UsageError(f"unknown option {flag}\n\n{USAGE}")
        if i + 1 >= len(argv) or argv[i + 1].startswith("--"):
            raise UsageError(f"{flag} requires a value")
        val = argv[i + 1]
        if flag == "--tris":
            cfg.triangles = num(flag, val)
        elif flag == "--iters":
            cfg.iters = num(flag, val)
        elif flag == "--size":
            opts["size"] = num(flag, val)
        elif flag == "--seed":
            cfg.seed = num(flag, val)
        elif flag == "--export":
            opts["export"] = num(flag, val)
        elif flag == "--save-every":
            opts["save_every"] = num(flag, val)
        elif flag == "--patience":
            n = num(flag, val)
            cfg.patience = n if n > 0 else None
        elif flag == "--out":
            opts["out"] = val
        elif flag == "--checkpoint":
            opts["checkpoint"] = val
        elif flag == "--checkpoint-every":
            opts["checkpoint_every"] = num(flag, val)
        elif flag == "--resume":
            opts["resume"] = val
        i += 2
    if opts["size"] == 0:
        raise UsageError("--size must be greater than zero")
    if opts["export"] == 0:
        raise UsageError("--export must be greater than zero")
    cfg.validate()
    return target, cfg, opts


def load_target(path: str | None, size: int) -> np.ndarray:
    if path is None:
        return formats.synthetic_target(size)
    if not os.path.exists(path):
        raise UsageError(f"no such file: {path}")
    return formats.load_target(path, size)


def run(argv: list[str]) -> int:
    parsed = parse_args(argv)
    if parsed is None:
        print(USAGE)
        return 0
    target_path, cfg, o = parsed
    target = load_target(target_path, o["size"])
    h, w = target.shape[:2]
    out = o["out"]
    os.makedirs(out, exist_ok=True)
    frames = os.path.join(out, "frames")
    if o["save_every"] > 0:
        os.makedirs(frames, exist_ok=True)
    formats.write_png(os.path.join(out, "target.png"), target)
    print(f"fitting {cfg.triangles} triangles to {target_path or '<synthetic target>'} at "
          f"{w}x{h} for {cfg.iters} iters")

    stepwise = o["save_every"] > 0 or o["checkpoint"] or o["resume"]
    start = time.perf_counter()
    if stepwise:
        f = (Fitter.from_state(target, o["resume"]) if o["resume"] else Fitter(target, cfg))
        cfg = f.cfg
        while (s := f.step()) is not None:
            if not o["quiet"] and (s.iter % 100 == 0 or s.iter + 1 == cfg.iters):
                print(f"  iter {s.iter:>5}  loss {s.loss:.6f}  sigma {s.sigma:.5f}")
            if o["save_every"] > 0 and s.iter % o["save_every"] == 0:
                img = f.render_current(s.sigma).cpu().numpy()
                formats.write_png(os.path.join(frames, f"frame_{s.iter // o['save_every']:05d}.png"),
                                  img)
            if o["checkpoint"] and o["checkpoint_every"] > 0 and f.iter % o["checkpoint_every"] == 0:
                f.save(o["checkpoint"])
        if o["checkpoint"]:
            f.save(o["checkpoint"])
        report = f.report()
    else:
        report = fit(target, cfg)
        if not o["quiet"]:
            from .fit import sigma_at
            for i, loss in enumerate(report.losses):
                if i % 100 == 0 or i + 1 == cfg.iters:
                    print(f"  iter {i:>5}  loss {loss:.6f}  sigma {sigma_at(cfg, i):.5f}")
    elapsed = time.perf_counter() - start

    # Geometry is normalised: render the best scene at the export size with
    # sigma scaled to keep the same softness in pixels (bin/fit.rs:94-97).
    ew, eh = formats.scale_to(w, h, o["export"])
    sharp = float(np.float32(cfg.sigma_end) * np.float32(w) / np.float32(ew))
    img = _native.render(torch.from_numpy(report.params[None]).cuda(), eh, ew, sharp,
                         report.background)[0].cpu().numpy()
    formats.write_png(os.path.join(out, "fit.png"), img)
    with open(os.path.join(out, "loss.csv"), "w") as fh:
        fh.write(formats.loss_csv(report.losses))
    with open(os.path.join(out, "scene.json"), "w") as fh:
        fh.write(formats.scene_to_json(report.params, report.background))

    note = {StopReason.COMPLETED: "completed", StopReason.CONVERGED: "converged early",
            StopReason.DIVERGED: "DIVERGED — returning best scene so far"}[report.stop_reason]
    print(f"\n{note} in {elapsed:.2f}s after {len(report.losses)} iters\n"
          f"loss {report.initial_loss():.6f} -> {report.best_loss:.6f} "
          f"({report.improvement():.1f}x lower, best at iter {report.best_iter})\n"
          f"wrote {os.path.join(out, 'fit.png')}")
    return 0


def main() -> None:
    try:
        sys.exit(run(sys.argv[1:]))
    except (UsageError, ConfigError, OSError, ValueError) as e:
        print(f"error: {e}", file=sys.stderr)
        sys.exit(1)


if __name__ == "__main__":
    main()
