"""The fit loop on the GPU: FitConfig, Fitter, fit (crates/diffrast/src/fit.rs).

Two drivers over the same device kernels:
- ``fit(target, cfg)`` without a progress callback runs the whole loop as one
  CUDA graph (``dr_fit``): no host round trip per iteration.
- ``Fitter`` advances one iteration per ``step()``: the fused forward + MSE +
  backward kernel, the reference's stop logic on the host, then the fused Adam
  kernel with projection. It can be checkpointed (``state_dict`` /
  ``Fitter.from_state``) and resumed exactly, and it feeds ``fit`` when a
  progress callback wants every iteration (frames, logging).

Seeding follows fit.rs:356-385 (background = the target's mean colour, random
geometry, colours sampled from the target at each centroid, alpha in
[0.3, 0.7)). The geometry comes from numpy's PCG64 stream rather than the
reference's StdRng, which cannot be reproduced here.
"""

from __future__ import annotations

import dataclasses
import enum
import math

import numpy as np
import torch

from . import _native
from .scenes import seed_scene_geometry

F32 = np.float32


class StopReason(enum.IntEnum):
    """fit.rs:14-23."""
    COMPLETED = 0
    CONVERGED = 1
    DIVERGED = 2


class ConfigError(ValueError):
    """fit.rs:26-46: a configuration that cannot produce a sensible fit."""


@dataclasses.dataclass
class FitConfig:
    """fit.rs:48-91 FitConfig with its defaults."""
    triangles: int = 128
    iters: int = 1500
    sigma_start: float = 0.02
    sigma_end: float = 0.0015
    lr_pos: float = 0.004
    lr_color: float = 0.02
    lr_alpha: float = 0.01
    seed: int = 0
    patience: int | None = 250
    min_delta: float = 1e-7

    def validate(self) -> None:
        """fit.rs:100-122, with the reference's messages."""
        if self.triangles <= 0:
            raise ConfigError("triangles must be greater than zero")
        s0, s1 = F32(self.sigma_start), F32(self.sigma_end)
        if not (np.isfinite(s0) and np.isfinite(s1)) or s0 <= 0 or s1 <= 0:
            raise ConfigError("sigma_start and sigma_end must be positive and finite")
        if s0 < s1:
            raise ConfigError("sigma_start must be greater than or equal to sigma_end")
        for lr in (self.lr_pos, self.lr_color, self.lr_alpha):
            if not math.isfinite(lr) or lr <= 0:
                raise ConfigError("learning rates must be positive and finite")


@dataclasses.dataclass
class FitReport:
    """fit.rs:134-165: the best scene, every loss, why it stopped."""
    params: np.ndarray          # (T, 10) best parameters
    background: tuple
    losses: list
    stop_reason: StopReason
    best_iter: int
    best_loss: float

    def final_loss(self) -> float:
        return self.losses[-1] if self.losses else float("nan")

    def initial_loss(self) -> float:
        return self.losses[0] if self.losses else float("nan")

    def improvement(self) -> float:
        return float(F32(self.initial_loss()) / F32(self.best_loss))


@dataclasses.dataclass
class StepInfo:
    iter: int
    loss: float
    sigma: float


def sigma_at(cfg: FitConfig, i: int) -> float:
    """fit.rs:343-349 in f32: geometric anneal from sigma_start to sigma_end."""
    if cfg.iters <= 1:
        return float(F32(cfg.sigma_end))
    t = F32(i) / F32(cfg.iters - 1)
    s0, s1 = F32(cfg.sigma_start), F32(cfg.sigma_end)
    return float(s0 * np.power(s1 / s0, t, dtype=np.float32))


def mean_color(target: np.ndarray) -> tuple:
    """fit.rs:370-379: f64 sum per channel, divided by the pixel count, as f32."""
    t = np.asarray(target, dtype=np.float32).reshape(-1, 3)
    n = float(F32(t.shape[0]))
    s = t.astype(np.float64).sum(axis=0)
    return tuple(float(F32(x / n)) for x in s)


def seed_colors(target: np.ndarray, params: np.ndarray) -> None:
    """fit.rs:361-366 + 381-385: each triangle's colour is the target's
    nearest pixel at its centroid (f32 centroid, truncating cast, clamped)."""
    h, w = target.shape[0], target.shape[1]
    for tri in params:
        cx = (F32(tri[0]) + F32(tri[2]) + F32(tri[4])) / F32(3.0)
        cy = (F32(tri[1]) + F32(tri[3]) + F32(tri[5])) / F32(3.0)
        px = min(max(int(math.trunc(float(cx * F32(w)))), 0), w - 1)
        py = min(max(int(math.trunc(float(cy * F32(h)))), 0), h - 1)
        tri[6:9] = target[py, px]


def seed_scene(target: np.ndarray, cfg: FitConfig) -> tuple[np.ndarray, tuple]:
    """fit.rs:356-368: the initial (T, 10) parameters and the background."""
    params = seed_scene_geometry(cfg.triangles, cfg.seed)
    seed_colors(np.asarray(target, dtype=np.float32), params)
    return params, mean_color(target)


class Fitter:
    """fit.rs:196-340, one iteration per step(), on the GPU."""

    def __init__(self, target, cfg: FitConfig | None = None, init_params=None, background=None,
                 device=None):
        cfg = cfg or FitConfig()
        cfg.validate()
        tgt = torch.as_tensor(np.asarray(target, dtype=np.float32) if not
                              isinstance(target, torch.Tensor) else target)
        if tgt.dim() != 3 or tgt.shape[2] != 3:
            raise ValueError("target must be (H, W, 3)")
        dev = _native._resolve_device(torch.device(device) if device is not None else
                                      (tgt.device if tgt.is_cuda else None))
        self.cfg = cfg
        self.device = dev
        self.target = tgt.to(dev, torch.float32).contiguous()
        if init_params is None:
            p, bg = seed_scene(self.target.cpu().numpy(), cfg)
        else:
            p = np.asarray(init_params, dtype=np.float32).reshape(-1, 10)
            bg = background if background is not None else mean_color(self.target.cpu().numpy())
        self.background = tuple(float(F32(x)) for x in bg)
        self.params = torch.from_numpy(np.ascontiguousarray(p)).to(dev)
        self.m = torch.zeros_like(self.params)
        self.v = torch.zeros_like(self.params)
        self.best_params = self.params.clone()
        self.losses: list[float] = []
        self.iter = 0
        self.since_improved = 0
        self.best_iter = 0
        self.best_loss = float("inf")
        self.stop_reason: StopReason | None = None

    def step(self) -> StepInfo | None:
        """fit.rs:243-288. None once the fit has stopped."""
        if self.stop_reason is not None:
            return None
        if self.iter >= self.cfg.iters:
            self.stop_reason = StopReason.COMPLETED
            return None
        i = self.iter
        sigma = sigma_at(self.cfg, i)
        losses, grads = _native.loss_backward(self.params[None], self.target[None], sigma,
                                              self.background)
        loss = float(losses[0].item())
        if not math.isfinite(loss):
            self.stop_reason = StopReason.DIVERGED
            return None
        self.losses.append(loss)
        if F32(loss) + F32(self.cfg.min_delta) < F32(self.best_loss):
            self.best_loss = loss
            self.best_iter = i
            self.best_params.copy_(self.params)
            self.since_improved = 0
        else:
            self.since_improved += 1
        self.iter += 1
        if self.cfg.patience is not None and self.since_improved >= self.cfg.patience:
            self.stop_reason = StopReason.CONVERGED
            return StepInfo(i, loss, sigma)
        _native.adam_step(self.params, self.m, self.v, grads[0].contiguous(), i + 1,
                          self.cfg.lr_pos, self.cfg.lr_color, self.cfg.lr_alpha, project=True)
        return StepInfo(i, loss, sigma)

    def is_done(self) -> bool:
        return self.stop_reason is not None or self.iter >= self.cfg.iters

    def sigma(self) -> float:
        """fit.rs:318-321: softness for the next iteration."""
        return sigma_at(self.cfg, min(self.iter, max(self.cfg.iters - 1, 0)))

    def render_current(self, sigma: float | None = None) -> torch.Tensor:
        """fit.rs:323-327: the current scene at sigma_end (H, W, 3)."""
        h, w = self.target.shape[0], self.target.shape[1]
        s = self.cfg.sigma_end if sigma is None else sigma
        return _native.render(self.params[None], h, w, s, self.background)[0]

    def report(self) -> FitReport:
        """fit.rs:329-338 into_report."""
        return FitReport(self.best_params.cpu().numpy(), self.background, list(self.losses),
                         self.stop_reason if self.stop_reason is not None else
                         StopReason.COMPLETED, self.best_iter, self.best_loss)

    # --- checkpoint / resume ------------------------------------------------------

    def state_dict(self) -> dict:
        """Everything the next step() depends on, as host arrays."""
        c = self.cfg
        return {
            "params": self.params.cpu().numpy(), "m": self.m.cpu().numpy(),
            "v": self.v.cpu().numpy(), "best_params": self.best_params.cpu().numpy(),
            "losses": np.asarray(self.losses, dtype=np.float64),
            "counters": np.asarray([self.iter, self.since_improved, self.best_iter,
                                    -1 if self.stop_reason is None else int(self.stop_reason)],
                                   dtype=np.int64),
            "best_loss": np.float64(self.best_loss),
            "background": np.asarray(self.background, dtype=np.float32),
            "cfg": np.asarray([c.triangles, c.iters, c.sigma_start, c.sigma_end, c.lr_pos,
                               c.lr_color, c.lr_alpha, c.seed,
                               -1 if c.patience is None else c.patience, c.min_delta],
                              dtype=np.float64),
        }

    def save(self, path) -> None:
        np.savez(path, **self.state_dict())

    @classmethod
    def from_state(cls, target, state, device=None) -> "Fitter":
        """Rebuild a Fitter from state_dict() output (or a file saved by save())."""
        if not isinstance(state, dict):
            with np.load(state) as z:
                state = {k: z[k] for k in z.files}
        c = state["cfg"]
        cfg = FitConfig(int(c[0]), int(c[1]), float(F32(c[2])), float(F32(c[3])),
                        float(F32(c[4])), float(F32(c[5])), float(F32(c[6])), int(c[7]),
                        None if c[8] < 0 else int(c[8]), float(F32(c[9])))
        f = cls(target, cfg, init_params=state["params"], background=state["background"],
                device=device)
        f.m.copy_(torch.from_numpy(state["m"]))
        f.v.copy_(torch.from_numpy(state["v"]))
        f.best_params.copy_(torch.from_numpy(state["best_params"]))
        f.losses = [float(x) for x in state["losses"]]
        it, since, best_iter, stop = (int(x) for x in state["counters"])
        f.iter, f.since_improved, f.best_iter = it, since, best_iter
        f.stop_reason = None if stop < 0 else StopReason(stop)
        f.best_loss = float(state["best_loss"])
        return f


def fit(target, cfg: FitConfig | None = None, progress=None, init_params=None,
        background=None) -> FitReport:
    """fit.rs:166-181. Without ``progress`` the loop runs as one CUDA graph
    (dr_fit); with it, ``progress(step_info, fitter)`` is called each iteration."""
    cfg = cfg or FitConfig()
    cfg.validate()
    if progress is not None:
        f = Fitter(target, cfg, init_params, background)
        while (s := f.step()) is not None:
            progress(s, f)
        return f.report()
    tgt = np.asarray(target.cpu() if isinstance(target, torch.Tensor) else target, np.float32)
    if init_params is None:
        p, bg = seed_scene(tgt, cfg)
    else:
        p = np.asarray(init_params, dtype=np.float32).reshape(-1, 10)
        bg = background if background is not None else mean_color(tgt)
    r = _native.fit(torch.from_numpy(tgt).cuda(), torch.from_numpy(p), bg, cfg.iters,
                    cfg.sigma_start, cfg.sigma_end, cfg.lr_pos, cfg.lr_color, cfg.lr_alpha,
                    cfg.patience, cfg.min_delta)
    return FitReport(np.asarray(r["best_params"].cpu() if isinstance(r["best_params"], torch.Tensor)
                                else r["best_params"], dtype=np.float32).reshape(-1, 10),
                     tuple(float(F32(x)) for x in bg), [float(x) for x in r["losses"]],
                     StopReason(int(r["stop_reason"])), int(r["best_iter"]), float(r["best_loss"]))
