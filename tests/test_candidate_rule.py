"""The block classification's candidate-edge pruning, checked on the CPU.

The raster kernels evaluate, per 8x4 warp block and triangle, only the
"candidate" edges of the block. In a block inside all three edge lines, an
edge is dropped when its line lies farther from every pixel than the smallest
per-edge maximum of the line distance (an upper bound of every pixel's nearest
segment distance there). This restates that rule in numpy and checks, pixel by pixel
over random triangles, sigmas and blocks, that the reference's nearest edge
(f32 segment distances, strict < in edge order, raster.rs:124-134,
grad.rs:236-242) is always a kept candidate wherever the pair composites and
is not deep inside.
"""

from __future__ import annotations

import numpy as np

f32 = np.float32


def make_edges(v):
    """Unit inward normals and line offsets computed in double and stored as
    f32 (as the set-up kernel does), the rounding margin and the winding sign."""
    v = v.astype(np.float64)
    area2 = (v[1, 0] - v[0, 0]) * (v[2, 1] - v[0, 1]) - (v[1, 1] - v[0, 1]) * (v[2, 0] - v[0, 0])
    s = 1.0 if area2 >= 0 else -1.0
    n = np.zeros((3, 2), np.float32)
    c = np.zeros(3, np.float32)
    for k in range(3):
        a, b = v[k], v[(k + 1) % 3]
        ex, ey = b - a
        ln = np.hypot(ex, ey)
        nx, ny = s * -ey / ln, s * ex / ln
        n[k] = (nx, ny)
        c[k] = -(nx * a[0] + ny * a[1])
    maxabs = np.abs(v).max()
    margin = f32(4e-6 * (2.0 + maxabs))
    return n, c, margin, s


def seg_ref(p, a, b):
    """point_segment_distance in f32 (raster.rs:124-134) and the cross product."""
    ex, ey = f32(b[0] - a[0]), f32(b[1] - a[1])
    apx, apy = f32(p[..., 0] - a[0]), f32(p[..., 1] - a[1])
    len2 = f32(f32(ex * ex) + f32(ey * ey))
    t = np.clip(f32(f32(f32(apx * ex) + f32(apy * ey)) / len2), f32(0), f32(1))
    dx, dy = f32(apx - f32(t * ex)), f32(apy - f32(t * ey))
    d = np.sqrt(f32(f32(dx * dx) + f32(dy * dy)))
    cross = f32(f32(ex * apy) - f32(ey * apx))
    return d, cross


def classify(v, n, c, margin, rej, acc, bx0, by0, W, H):
    inv_w, inv_h = f32(1.0 / W), f32(1.0 / H)
    cx, hx = f32(0.5 * (2 * bx0 + 8) * inv_w), f32(0.5 * 7 * inv_w)
    cy, hy = f32(0.5 * (2 * by0 + 4) * inv_h), f32(0.5 * 3 * inv_h)
    thr = max(rej, acc) + margin
    lmin, lmax, cand = np.zeros(3, np.float32), np.zeros(3, np.float32), 0
    for e in range(3):
        lc = n[e, 0] * cx + n[e, 1] * cy + c[e]
        rad = abs(n[e, 0]) * hx + abs(n[e, 1]) * hy
        if lc + rad < -rej:
            return "skip", 0, 0
        lmin[e], lmax[e] = lc - rad, lc + rad
        if not (abs(lc) - rad > thr):
            cand |= 1 << e
    if lmin.min() > acc:
        return "inside", 0, 0
    before = cand
    if cand & (cand - 1) and lmin.min() > margin:
        lim = lmax.min() + 2 * margin
        for e in range(3):
            if lmin[e] > lim:
                cand &= ~(1 << e)
    return "cand", cand, before


def test_pruned_candidates_always_hold_the_nearest_edge():
    rng = np.random.default_rng(11)
    W = H = 256
    checked = pruned = 0
    for _ in range(400):
        v = rng.uniform(0.1, 0.9, size=(3, 2)).astype(np.float32)
        if rng.uniform() < 0.5:  # small and thin triangles too
            v = (v[0] + (v - v[0]) * rng.uniform(0.05, 0.4)).astype(np.float32)
        n, c, margin, wind = make_edges(v)
        e0 = v[1] - v[0]
        e2 = v[2] - v[0]
        if abs(e0[0] * e2[1] - e0[1] * e2[0]) < 1e-6:
            continue
        sigma = f32(rng.choice([0.0015, 0.005, 0.01, 0.02]))
        alpha = rng.uniform(0.2, 1.0)
        rej = f32((max(np.log(alpha * 1e6), 0.0) + 0.2) * sigma) + margin
        acc = f32(16.8 * sigma) + margin
        lo = np.floor((v.min(0) - 6 * sigma) * W).astype(int)
        hi = np.ceil((v.max(0) + 6 * sigma) * W).astype(int)
        for _ in range(12):
            bx0 = int(rng.integers(max(lo[0], 0), min(hi[0], W - 8) + 1)) // 8 * 8
            by0 = int(rng.integers(max(lo[1], 0), min(hi[1], H - 4) + 1)) // 4 * 4
            kind, cand, before = classify(v, n, c, margin, rej, acc, bx0, by0, W, H)
            if kind != "cand":
                continue
            pruned += cand != before
            xs = (np.arange(bx0, bx0 + 8, dtype=np.float32) + f32(0.5)) / f32(W)
            ys = (np.arange(by0, by0 + 4, dtype=np.float32) + f32(0.5)) / f32(H)
            p = np.stack(np.meshgrid(xs, ys), -1).reshape(-1, 2).astype(np.float32)
            d = np.zeros((3, len(p)), np.float32)
            cr = np.zeros((3, len(p)), np.float32)
            for e in range(3):
                d[e], cr[e] = seg_ref(p, v[e], v[(e + 1) % 3])
            nearest = np.argmin(d, axis=0)  # first minimum: the reference's strict <
            inside = np.all(cr >= 0, 0) | np.all(cr <= 0, 0)
            best = d.min(0)
            sd = np.where(inside, best, -best)
            matters = (sd / sigma < 16.8) & (sd > -rej)
            for i in np.nonzero(matters)[0]:
                checked += 1
                assert cand & (1 << int(nearest[i])), (v, sigma, bx0, by0, cand, i)
    # Pixels checked, and blocks where the rule dropped an edge.
    assert checked > 2000 and pruned > 30, (checked, pruned)
