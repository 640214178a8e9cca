"""ctypes wrapper around the CPU oracle (``oracle/diffrast_oracle.cpp``).

TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline. The
product (``differentiable-rasterizer_b200/``) never imports this package; only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs do.

The C++ it wraps restates the reference's Rust CPU path
(crates/diffrast/src/raster.rs:26-168, grad.rs:56-323, canvas.rs:45-59,
optim.rs:40-60, fit.rs:243-424, diffrast-py/src/lib.rs:301-318). Every
function here takes and returns numpy arrays in the reference's layouts:
params ``(B, T, 10)`` as ``[x0, y0, x1, y1, x2, y2, r, g, b, a]`` and images
``(B, H, W, 3)``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdiffrast_oracle.so")

MODE_TARGET = 0  # d_canvas = 2/N (r - t)            (grad.rs:112-114)
MODE_INVERT_GRAD = 1  # t = r - g*N/2, then MODE_TARGET (diffrast-py lib.rs:311-313)
MODE_DIRECT_GRAD = 2  # d_canvas = upstream gradient    (backward_batch_reduced.wgsl:146-147)

STOP_COMPLETED, STOP_CONVERGED, STOP_DIVERGED = 0, 1, 2


def build(force: bool = False) -> str:
    """Compile the oracle library with ``oracle/Makefile`` (g++ only)."""
    src = os.path.join(_HERE, "diffrast_oracle.cpp")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return LIB_PATH


_lib = None

_F = ctypes.POINTER(ctypes.c_float)
_D = ctypes.POINTER(ctypes.c_double)
_I64 = ctypes.POINTER(ctypes.c_int64)
_U32 = ctypes.POINTER(ctypes.c_uint32)
_I = ctypes.c_int
_I64V = ctypes.c_int64
_FV = ctypes.c_float


class FitConfigC(ctypes.Structure):
    _fields_ = [
        ("iters", ctypes.c_int64),
        ("sigma_start", ctypes.c_float),
        ("sigma_end", ctypes.c_float),
        ("lr_pos", ctypes.c_float),
        ("lr_color", ctypes.c_float),
        ("lr_alpha", ctypes.c_float),
        ("patience", ctypes.c_int64),
        ("min_delta", ctypes.c_float),
    ]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        sig = {
            "oracle_pixel_bounds": (_I, [_F, _I, _I, _FV, _I64]),
            "oracle_signed_distance": (_FV, [_F, _FV, _FV]),
            "oracle_coverage": (_FV, [_F, _FV, _FV, _FV]),
            "oracle_coverage_with_grad": (_FV, [_F, _FV, _FV, _FV, _F]),
            "oracle_mse": (_FV, [_F, _F, _I64V]),
            "oracle_render_batch": (None, [_F, _F, _I, _I, _I, _I, _I, _FV, _F, _I]),
            "oracle64_render_batch": (None, [_F, _F, _I, _I, _I, _I, _I, _FV, _D, _I]),
            "oracle_backward_batch": (
                None,
                [_F, _F, _I, _I, _I, _I, _I, _FV, _F, _I, _F, _F, _F, _I],
            ),
            "oracle64_backward_batch": (
                None,
                [_F, _F, _I, _I, _I, _I, _I, _FV, _F, _I, _D, _D, _D, _I],
            ),
            "oracle_finite_difference": (_FV, [_F, _F, _I, _I, _I, _FV, _F, _FV, _F]),
            "oracle_powi": (_FV, [_FV, _I]),
            "oracle_adam_step": (None, [_F, _F, _F, _F, _F, _I64V, _U32, _FV, _FV, _FV]),
            "oracle_project": (None, [_F, _I64V]),
            "oracle_sigma_at": (_FV, [_FV, _FV, _I64V, _I64V]),
            "oracle_seed_colors": (None, [_F, _I, _I, _F, _I, _F]),
            "oracle_fit_validate": (_I, [ctypes.POINTER(FitConfigC), _I]),
            "oracle_fit": (
                _I,
                [_F, _I, _I, _F, _F, _I, ctypes.POINTER(FitConfigC), _F, _I64, _F, _F, _I64, _F,
                 ctypes.POINTER(ctypes.c_int)],
            ),
            "oracle64_fit": (
                _I,
                [_F, _I, _I, _F, _F, _I, ctypes.POINTER(FitConfigC), _D, _I64, _D, _D, _I64, _D,
                 ctypes.POINTER(ctypes.c_int)],
            ),
            "oracle_num_threads": (_I, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a: np.ndarray):
    if a.dtype == np.float32:
        return a.ctypes.data_as(_F)
    if a.dtype == np.float64:
        return a.ctypes.data_as(_D)
    raise TypeError(a.dtype)


def _bg(background, batch: int):
    bg = _f32(background)
    if bg.size == 3:
        return bg.reshape(3), 0
    if bg.shape != (batch, 3):
        raise ValueError("background must be 3 values or (B, 3)")
    return bg.reshape(-1), 1


def num_threads() -> int:
    return lib().oracle_num_threads()


# --- geometry probes --------------------------------------------------------


def pixel_bounds(tri, width: int, height: int, sigma: float):
    out = np.zeros(4, dtype=np.int64)
    t = _f32(tri)
    ok = lib().oracle_pixel_bounds(_p(t), width, height, sigma, out.ctypes.data_as(_I64))
    return tuple(int(v) for v in out) if ok else None


def signed_distance(verts, pt) -> float:
    v = _f32(verts).reshape(6)
    return lib().oracle_signed_distance(_p(v), float(pt[0]), float(pt[1]))


def coverage(tri, pt, sigma: float) -> float:
    t = _f32(tri)
    return lib().oracle_coverage(_p(t), float(pt[0]), float(pt[1]), sigma)


def coverage_with_grad(tri, pt, sigma: float):
    t = _f32(tri)
    d = np.zeros(6, dtype=np.float32)
    cov = lib().oracle_coverage_with_grad(_p(t), float(pt[0]), float(pt[1]), sigma, _p(d))
    return cov, d


def mse(a, b) -> float:
    a, b = _f32(a), _f32(b)
    assert a.size == b.size
    return lib().oracle_mse(_p(a), _p(b), a.size)


# --- batched path -----------------------------------------------------------


def render_batch(params, height: int, width: int, sigma: float, background=(0.0, 0.0, 0.0),
                 threads: int = 0, f64: bool = False) -> np.ndarray:
    """raster.rs:37-68 over a batch (grad.rs:210-212). Returns (B, H, W, 3)."""
    p = _f32(params)
    B, T, n = p.shape
    assert n == 10
    bg, per = _bg(background, B)
    if f64:
        out = np.empty((B, height, width, 3), dtype=np.float64)
        lib().oracle64_render_batch(_p(p), _p(bg), per, B, T, height, width, sigma, _p(out),
                                    threads)
    else:
        out = np.empty((B, height, width, 3), dtype=np.float32)
        lib().oracle_render_batch(_p(p), _p(bg), per, B, T, height, width, sigma, _p(out),
                                  threads)
    return out


def backward_batch(params, other, sigma: float, background=(0.0, 0.0, 0.0), mode=MODE_TARGET,
                   threads: int = 0, f64: bool = False, want_images: bool = False):
    """render_with_tape + backward per scene (grad.rs:192-207).

    ``other`` is the (B, H, W, 3) target (``MODE_TARGET``) or upstream image
    gradient (``MODE_INVERT_GRAD`` / ``MODE_DIRECT_GRAD``). Returns
    ``(losses (B,), grads (B, T, 10)[, images (B, H, W, 3)])``.
    """
    p = _f32(params)
    o = _f32(other)
    B, T, n = p.shape
    assert n == 10 and o.ndim == 4 and o.shape[0] == B and o.shape[3] == 3
    H, W = o.shape[1], o.shape[2]
    bg, per = _bg(background, B)
    dt = np.float64 if f64 else np.float32
    losses = np.zeros(B, dtype=dt)
    grads = np.zeros((B, T, 10), dtype=dt)
    images = np.zeros((B, H, W, 3), dtype=dt) if want_images else None
    fn = lib().oracle64_backward_batch if f64 else lib().oracle_backward_batch
    fn(_p(p), _p(bg), per, B, T, H, W, sigma, _p(o), mode, _p(losses), _p(grads),
       _p(images) if want_images else None, threads)
    if want_images:
        return losses, grads, images
    return losses, grads


def finite_difference(params, height: int, width: int, sigma: float, target,
                      background=(0.0, 0.0, 0.0), eps: float = 1e-3):
    """grad.rs:298-323 for one scene ((T, 10) params). Returns (loss, grads)."""
    p = _f32(params)
    T = p.shape[0]
    t = _f32(target)
    bg = _f32(background).reshape(3)
    g = np.zeros((T, 10), dtype=np.float32)
    loss = lib().oracle_finite_difference(_p(p), _p(bg), T, height, width, sigma, _p(t), eps,
                                          _p(g))
    return loss, g


# --- optimizer / fit ---------------------------------------------------------


def powi(a: float, b: int) -> float:
    return lib().oracle_powi(a, b)


class Adam:
    """optim.rs:11-60 over a flat f32 vector."""

    def __init__(self, n: int, beta1=0.9, beta2=0.999, eps=1e-8):
        self.m = np.zeros(n, dtype=np.float32)
        self.v = np.zeros(n, dtype=np.float32)
        self.t = ctypes.c_uint32(0)
        self.beta1, self.beta2, self.eps = beta1, beta2, eps

    @property
    def steps_taken(self) -> int:
        return self.t.value

    def step(self, params: np.ndarray, grads, lr) -> None:
        assert params.dtype == np.float32 and params.flags.c_contiguous
        g, l = _f32(grads), _f32(lr)
        assert g.size == params.size and l.size == params.size
        lib().oracle_adam_step(_p(params), _p(self.m), _p(self.v), _p(g), _p(l), params.size,
                               ctypes.byref(self.t), self.beta1, self.beta2, self.eps)


def project(params: np.ndarray) -> None:
    assert params.dtype == np.float32 and params.flags.c_contiguous and params.size % 10 == 0
    lib().oracle_project(_p(params), params.size // 10)


def sigma_at(sigma_start: float, sigma_end: float, iters: int, i: int) -> float:
    return lib().oracle_sigma_at(sigma_start, sigma_end, iters, i)


def learning_rates(n_tris: int, lr_pos=0.004, lr_color=0.02, lr_alpha=0.01) -> np.ndarray:
    """fit.rs:388-396"""
    row = np.array([lr_pos] * 6 + [lr_color] * 3 + [lr_alpha], dtype=np.float32)
    return np.tile(row, n_tris)


def seed_colors(target, params):
    """fit.rs:356-385 colour/background part of seed_scene (in place on params)."""
    t = _f32(target)
    H, W = t.shape[0], t.shape[1]
    p = params
    assert p.dtype == np.float32 and p.flags.c_contiguous
    bg = np.zeros(3, dtype=np.float32)
    lib().oracle_seed_colors(_p(t), H, W, _p(p), p.size // 10, _p(bg))
    return bg


@dataclass
class FitConfig:
    """fit.rs:49-89 defaults (the `triangles`/`seed` fields come from the init)."""

    iters: int = 1500
    sigma_start: float = 0.02
    sigma_end: float = 0.0015
    lr_pos: float = 0.004
    lr_color: float = 0.02
    lr_alpha: float = 0.01
    patience: int | None = 250
    min_delta: float = 1e-7

    def c(self) -> FitConfigC:
        return FitConfigC(self.iters, self.sigma_start, self.sigma_end, self.lr_pos, self.lr_color,
                          self.lr_alpha, -1 if self.patience is None else self.patience,
                          self.min_delta)


CONFIG_ERRORS = {1: "NoTriangles", 2: "NonPositiveSigma", 3: "SigmaNotDecreasing",
                 4: "NonPositiveLearningRate"}


@dataclass
class FitReport:
    losses: np.ndarray
    best_params: np.ndarray
    final_params: np.ndarray
    best_iter: int
    best_loss: float
    stop_reason: int


def fit(target, init_params, background, cfg: FitConfig, f64: bool = False) -> FitReport:
    """fit.rs:166-181 from a given seeded scene; raises ValueError(ConfigError).

    ``f64=True`` runs the twin that carries parameters, Adam moments and the
    loss in f64 (the sigma schedule and box cull stay f32): the spread between
    the two is the f32 rounding noise floor of a fit."""
    t = _f32(target)
    H, W = t.shape[0], t.shape[1]
    p = _f32(init_params).reshape(-1, 10)
    T = p.shape[0]
    bg = _f32(background).reshape(3)
    dt = np.float64 if f64 else np.float32
    losses = np.zeros(max(cfg.iters, 1), dtype=dt)
    n_losses = ctypes.c_int64(0)
    best = np.zeros(p.shape, dtype=dt)
    final = np.zeros(p.shape, dtype=dt)
    bi = ctypes.c_int64(0)
    bl = ctypes.c_double(0) if f64 else ctypes.c_float(0)
    stop = ctypes.c_int(0)
    c = cfg.c()
    fn = lib().oracle64_fit if f64 else lib().oracle_fit
    err = fn(_p(t), H, W, _p(p), _p(bg), T, ctypes.byref(c), _p(losses),
             ctypes.byref(n_losses), _p(best), _p(final), ctypes.byref(bi),
             ctypes.byref(bl), ctypes.byref(stop))
    if err:
        raise ValueError(CONFIG_ERRORS[err])
    return FitReport(losses[: n_losses.value].copy(), best, final, bi.value, bl.value, stop.value)
