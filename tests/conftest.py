"""Shared test set-up.

Markers: ``gpu`` tests need a CUDA device (run on a B200 with ``-m gpu``); all
other tests run on CPU only. The CPU oracle (``oracle/``) is the parity checker.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "differentiable-rasterizer_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available() and torch.cuda.device_count() > 0
    except Exception:
        return False


@pytest.fixture(scope="session")
def oracle():
    import oracle as o

    o.build()
    return o


# --- parity tolerances (images 1e-5 abs + 1e-4 rel, gradients 1e-6 + 1e-3 rel) --

IMAGE_ATOL = 1e-5
IMAGE_RTOL = 1e-4
GRAD_ATOL = 1e-6
GRAD_RTOL = 1e-3


def assert_images_close(got, ref, what="image"):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    nan_got, nan_ref = np.isnan(got), np.isnan(ref)
    assert np.array_equal(nan_got, nan_ref), f"{what}: NaN pattern differs"
    g, r = got[~nan_ref], ref[~nan_ref]
    err = np.abs(g - r)
    bad = err > IMAGE_ATOL + IMAGE_RTOL * np.abs(r)
    assert not bad.any(), (
        f"{what}: {bad.sum()} of {bad.size} values outside |d| <= {IMAGE_ATOL} + "
        f"{IMAGE_RTOL}|ref| (max |d| {err.max():.3e})")


def assert_grads_close(got, ref, what="grads", slack=None):
    """Per-element |d| <= 1e-6 + 1e-3 |ref| (+ an optional per-element slack,
    the f32-vs-f64 oracle spread, for cancellation-dominated entries)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    nan_got, nan_ref = np.isnan(got), np.isnan(ref)
    assert np.array_equal(nan_got, nan_ref), f"{what}: NaN pattern differs"
    g, r = got[~nan_ref], ref[~nan_ref]
    tol = GRAD_ATOL + GRAD_RTOL * np.abs(r)
    if slack is not None:
        tol = tol + np.asarray(slack, dtype=np.float64)[~nan_ref]
    err = np.abs(g - r)
    bad = err > tol
    if bad.any():
        i = np.argmax(err - tol)
        raise AssertionError(
            f"{what}: {bad.sum()} of {bad.size} elements outside tolerance; worst "
            f"got {g[i]:.6e} ref {r[i]:.6e} |d| {err[i]:.3e} tol {tol[i]:.3e}")


def rel_norm_error(got, ref) -> float:
    """The reference's own metric, max|d| / ||ref||_2 (diffrast-gpu lib.rs:1252-1254)."""
    got = np.asarray(got, dtype=np.float64).ravel()
    ref = np.asarray(ref, dtype=np.float64).ravel()
    return float(np.max(np.abs(got - ref)) / max(np.linalg.norm(ref), 1e-12))
