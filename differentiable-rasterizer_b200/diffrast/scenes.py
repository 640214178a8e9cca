"""Seeded synthetic scenes for the benchmark configurations.

The reference publishes no dataset for this path; its benchmarks draw random
scenes (benches/raster.rs:16-19, gpu_bench.rs:18-21, Scene::random
scene.rs:58-76). These generators reproduce the *shapes and distributions* of
the five benchmark configurations with numpy's PCG64 (the reference's StdRng
stream cannot be reproduced without its Rust dependencies), so the GPU path,
the CPU oracle and the bench all consume identical bytes.

All params are float32 ``(B, T, 10)`` = ``[x0, y0, x1, y1, x2, y2, r, g, b, a]``.
"""

from __future__ import annotations

import math

import numpy as np


def uniform_scenes(batch: int, tris: int, seed: int, opacity=(0.2, 1.0),
                   lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
    """Vertices U[lo,hi]^2, RGB U[0,1], opacity U[opacity]. Per scene the draw
    order is verts (T x 6), rgb (T x 3), opacity (T)."""
    rng = np.random.default_rng(seed)
    out = np.empty((batch, tris, 10), dtype=np.float32)
    for b in range(batch):
        out[b, :, 0:6] = rng.uniform(lo, hi, size=(tris, 6))
        out[b, :, 6:9] = rng.uniform(0.0, 1.0, size=(tris, 3))
        out[b, :, 9] = rng.uniform(opacity[0], opacity[1], size=tris)
    return out


def config2_params(batch: int, tris: int, cell: int) -> tuple[np.ndarray, np.ndarray]:
    """Config 2 grid cell: (params seed 2000+cell, target-scene params seed 3000+cell)."""
    return (uniform_scenes(batch, tris, 2000 + cell),
            uniform_scenes(batch, tris, 3000 + cell))


def seed_scene_geometry(tris: int, seed: int, seed_scale: float = 0.18) -> np.ndarray:
    """Geometry/alpha part of fit.rs:356-367 seed_scene with PCG64: centroid
    U[0,1)^2 plus U(-0.18, 0.18) per vertex coordinate, alpha U[0.3, 0.7).
    Colours are left at 0; the fit's seed_colors fills them from the target."""
    rng = np.random.default_rng(seed)
    out = np.zeros((tris, 10), dtype=np.float32)
    for k in range(tris):
        cx, cy = rng.uniform(0.0, 1.0, size=2)
        for v in range(3):
            out[k, 2 * v] = cx + rng.uniform(-seed_scale, seed_scale)
            out[k, 2 * v + 1] = cy + rng.uniform(-seed_scale, seed_scale)
        out[k, 9] = rng.uniform(0.3, 0.7)
    return out


def config1_target_scene(tris: int = 150, seed: int = 0) -> np.ndarray:
    """Config 1 target scene: verts U[0,1]^2, rgb U[0,1], opacity U[0.3,1]."""
    return uniform_scenes(1, tris, seed, opacity=(0.3, 1.0))


def config4_params(tris: int = 4096, seed: int = 4000) -> np.ndarray:
    """Config 4: equilateral triangles, area log-uniform in [1e-5, 1e-2],
    centre U[0,1]^2, rotation U[0, 2pi), rgb U[0,1], opacity U[0.2,1]."""
    rng = np.random.default_rng(seed)
    out = np.empty((1, tris, 10), dtype=np.float32)
    centre = rng.uniform(0.0, 1.0, size=(tris, 2))
    area = np.exp(rng.uniform(math.log(1e-5), math.log(1e-2), size=tris))
    rot = rng.uniform(0.0, 2 * math.pi, size=tris)
    rgb = rng.uniform(0.0, 1.0, size=(tris, 3))
    alpha = rng.uniform(0.2, 1.0, size=tris)
    side = np.sqrt(4.0 * area / math.sqrt(3.0))
    radius = side / math.sqrt(3.0)  # centroid-to-vertex distance
    for v in range(3):
        ang = rot + v * 2.0 * math.pi / 3.0
        out[0, :, 2 * v] = centre[:, 0] + radius * np.cos(ang)
        out[0, :, 2 * v + 1] = centre[:, 1] + radius * np.sin(ang)
    out[0, :, 6:9] = rgb
    out[0, :, 9] = alpha
    return out


def config5_params(batch: int = 16, tris: int = 2048, seed: int = 5000) -> np.ndarray:
    """Config 5 stress scenes: all vertices in [0.4, 0.6]^2; per scene 5%
    degenerate triangles (half collinear v2 = v0 + s (v1 - v0), s U[-0.5,1.5];
    half coincident v1 = v0, every 4th of those with all three equal); 2.5%
    opacity exactly 0 and 2.5% exactly 1; the rest U[0.2, 1]."""
    out = np.empty((batch, tris, 10), dtype=np.float32)
    for b in range(batch):
        rng = np.random.default_rng(seed + b)
        p = np.empty((tris, 10), dtype=np.float32)
        p[:, 0:6] = rng.uniform(0.4, 0.6, size=(tris, 6))
        p[:, 6:9] = rng.uniform(0.0, 1.0, size=(tris, 3))
        p[:, 9] = rng.uniform(0.2, 1.0, size=tris)
        idx = rng.permutation(tris)
        n_deg = int(round(0.05 * tris))
        deg = idx[:n_deg]
        half = n_deg // 2
        for j, k in enumerate(deg):
            if j < half:
                s = rng.uniform(-0.5, 1.5)
                p[k, 4] = p[k, 0] + s * (p[k, 2] - p[k, 0])
                p[k, 5] = p[k, 1] + s * (p[k, 3] - p[k, 1])
            else:
                p[k, 2] = p[k, 0]
                p[k, 3] = p[k, 1]
                if (j - half) % 4 == 0:
                    p[k, 4] = p[k, 0]
                    p[k, 5] = p[k, 1]
        n_a = int(round(0.025 * tris))
        p[idx[n_deg:n_deg + n_a], 9] = 0.0
        p[idx[n_deg + n_a:n_deg + 2 * n_a], 9] = 1.0
        out[b] = p
    return out


def bbox_pairs(params: np.ndarray, width: int, height: int, sigma: float) -> int:
    """Bounding-box pairs of a batch, the roofline's unit of work: the pixels
    inside pixel_bounds (raster.rs:144-168, f32 arithmetic: 6 sigma of padding,
    floor / ceil + 1, clamped to the canvas) summed over the triangles with
    alpha > 0 and finite vertices."""
    p = np.asarray(params, dtype=np.float32).reshape(-1, 10)
    v = p[:, :6].reshape(-1, 3, 2)
    live = (p[:, 9] > 0) & np.isfinite(v).all(axis=(1, 2))
    v = v[live]
    if v.shape[0] == 0:
        return 0
    pad = np.float32(6.0) * np.float32(sigma)
    size = np.array([width, height], dtype=np.float32)
    lo = np.floor((v.min(axis=1) - pad) * size)
    hi = np.ceil((v.max(axis=1) + pad) * size)
    lim = np.float32(2.0 ** 62)  # far beyond any canvas: saturation is never reached
    x0y0 = np.minimum(np.maximum(lo, 0), lim).astype(np.int64)
    x1y1 = np.minimum(np.minimum(np.maximum(hi, 0), lim).astype(np.int64) + 1,
                      np.array([width, height], dtype=np.int64))
    ext = np.clip(x1y1 - x0y0, 0, None)
    return int((ext[:, 0] * ext[:, 1]).sum())
