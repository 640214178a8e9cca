"""Fit artefact formats and the fit CLI's host logic (CPU).

Restates the reference's own tests of these formats: serial.rs:85-117 (scene
JSON), canvas.rs:123-158 (sRGB, fit_within), fit.rs config validation, and
bin/fit.rs argument handling.
"""

from __future__ import annotations

import json
import os
import struct
import zlib

import numpy as np
import pytest


def sample_scene():
    """serial.rs:77-82."""
    return np.array([[0.0, 0.0, 1.0, 0.0, 0.5, 1.0, 1.0, 0.5, 0.25, 0.75]], np.float32), (0.1, 0.2,
                                                                                          0.3)


def test_json_emits_expected_fields():
    from diffrast.formats import scene_to_json

    p, bg = sample_scene()
    j = scene_to_json(p, bg)
    assert '"version": 1' in j
    assert '"background": [0.100000, 0.200000, 0.300000]' in j
    assert '"alpha": 0.750000' in j
    assert json.loads(j)["triangles"][0]["verts"] == [[0.0, 0.0], [1.0, 0.0], [0.5, 1.0]]


def test_json_empty_scene_is_still_valid():
    from diffrast.formats import scene_to_json

    j = scene_to_json(np.zeros((0, 10), np.float32), (0.0, 0.0, 0.0))
    assert '"triangles": [\n  ]' in j
    assert json.loads(j)["triangles"] == []


def test_json_non_finite_values_never_reach_the_output():
    from diffrast.formats import scene_to_json

    p, bg = sample_scene()
    p[0, 9] = np.nan
    p[0, 0] = np.inf
    j = scene_to_json(p, bg)
    assert "NaN" not in j and "inf" not in j
    json.loads(j)


def test_json_triangle_count_matches_separators():
    from diffrast.formats import scene_to_json

    p, bg = sample_scene()
    j = scene_to_json(np.repeat(p, 3, axis=0), bg)
    assert j.count('"verts"') == 3
    assert j.count("},\n") == 2


def test_json_whole_layout():
    from diffrast.formats import scene_to_json

    p, bg = sample_scene()
    assert scene_to_json(p, bg) == (
        '{\n  "version": 1,\n  "background": [0.100000, 0.200000, 0.300000],\n'
        '  "triangles": [\n'
        '    {"verts": [[0.000000, 0.000000], [1.000000, 0.000000], [0.500000, 1.000000]], '
        '"color": [1.000000, 0.500000, 0.250000], "alpha": 0.750000}\n  ]\n}\n')


def test_loss_csv_uses_rust_float_display():
    from diffrast.formats import loss_csv

    assert loss_csv([0.5, 1.0, 1e-7, 0.0123, float("nan"), float("inf")]) == (
        "iter,loss\n0,0.5\n1,1\n2,0.0000001\n3,0.0123\n4,NaN\n5,inf\n")
    # f32 shortest round-trip digits, not the f64 value's.
    assert loss_csv([0.1]) == "iter,loss\n0,0.1\n"


def test_srgb_round_trips_through_encode_decode():
    from diffrast.formats import decode_srgb, encode_srgb

    v = np.array([0, 1, 17, 128, 200, 255], np.uint8)
    assert np.array_equal(encode_srgb(decode_srgb(v)), v)


def test_out_of_range_values_are_clamped_when_encoding():
    from diffrast.formats import encode_srgb

    assert encode_srgb(np.float32(-1.0)) == 0
    assert encode_srgb(np.float32(2.0)) == 255
    assert encode_srgb(np.float32(np.nan)) == 0


def test_fit_within_preserves_aspect_and_never_upscales():
    from diffrast.formats import fit_within

    assert fit_within(1000, 500, 200) == (200, 100)
    assert fit_within(500, 1000, 200) == (100, 200)
    assert fit_within(64, 32, 200) == (64, 32)
    assert fit_within(0, 0, 200) == (1, 1)
    assert fit_within(10_000, 1, 100) == (100, 1)


def _png_with_filters(img: np.ndarray) -> bytes:
    """An RGB PNG whose rows use filter types 0..4 in turn (for the reader)."""
    h, w, _ = img.shape
    bpp = 3
    rows = []
    prev = np.zeros(w * 3, np.int32)
    for y in range(h):
        cur = img[y].reshape(-1).astype(np.int32)
        ft = y % 5
        out = np.empty_like(cur)
        for x in range(w * 3):
            a = cur[x - bpp] if x >= bpp else 0
            b = prev[x]
            c = prev[x - bpp] if x >= bpp else 0
            if ft == 0:
                pred = 0
            elif ft == 1:
                pred = a
            elif ft == 2:
                pred = b
            elif ft == 3:
                pred = (a + b) >> 1
            else:
                pa, pb, pc = abs(b - c), abs(a - c), abs(a + b - 2 * c)
                pred = a if (pa <= pb and pa <= pc) else (b if pb <= pc else c)
            out[x] = (cur[x] - pred) & 0xFF
        rows.append(bytes([ft]) + out.astype(np.uint8).tobytes())
        prev = cur

    def chunk(k, d):
        return struct.pack(">I", len(d)) + k + d + struct.pack(">I", zlib.crc32(k + d))

    return (b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, 8, 2, 0, 0, 0)) +
            chunk(b"IDAT", zlib.compress(b"".join(rows))) + chunk(b"IEND", b""))


def test_png_round_trip_and_all_filter_types(tmp_path):
    from diffrast.formats import read_png, write_png, decode_srgb, encode_srgb

    rng = np.random.default_rng(0)
    img = rng.integers(0, 256, size=(11, 7, 3), dtype=np.uint8)
    path = tmp_path / "f.png"
    path.write_bytes(_png_with_filters(img))
    assert np.array_equal(read_png(path), img)
    lin = decode_srgb(img)
    write_png(tmp_path / "g.png", lin)
    assert np.array_equal(read_png(tmp_path / "g.png"), encode_srgb(lin))


def test_lanczos_resize_keeps_flat_images_flat_and_shapes():
    from diffrast.formats import resize_lanczos3

    flat = np.full((40, 30, 3), 77, np.uint8)
    assert np.array_equal(resize_lanczos3(flat, 12, 16), np.full((16, 12, 3), 77, np.uint8))
    grad = np.tile(np.arange(64, dtype=np.uint8)[None, :, None] * 4, (8, 1, 3))
    small = resize_lanczos3(grad, 16, 8)
    assert small.shape == (8, 16, 3)
    assert np.all(np.diff(small[4, :, 0].astype(int)) >= 0)


def test_synthetic_target_matches_the_oracle_coverage(oracle):
    # bin/fit.rs:219-250, recomputed here with the oracle's coverage().
    from diffrast.formats import synthetic_target

    size = 24
    got = synthetic_target(size)
    ref = np.empty_like(got)
    for y in range(size):
        for x in range(size):
            u, v = np.float32(x) / np.float32(size), np.float32(y) / np.float32(size)
            ref[y, x] = [np.float32(0.15) + np.float32(0.5) * u, np.float32(0.10) +
                         np.float32(0.4) * v, np.float32(0.55) - np.float32(0.3) * u]
    shapes = [([[0.15, 0.70], [0.55, 0.68], [0.35, 0.20]], [0.95, 0.85, 0.25]),
              ([[0.50, 0.30], [0.88, 0.45], [0.62, 0.85]], [0.10, 0.25, 0.45])]
    for verts, col in shapes:
        t = np.array(sum(verts, []) + col + [1.0], np.float32)
        for y in range(size):
            for x in range(size):
                pt = ((np.float32(x) + np.float32(0.5)) / np.float32(size),
                      (np.float32(y) + np.float32(0.5)) / np.float32(size))
                w = np.float32(oracle.coverage(t, pt, 0.002))
                if w <= np.float32(1e-4):
                    continue
                ref[y, x] = [np.float32(col[c]) * w + ref[y, x, c] * (np.float32(1.0) - w)
                             for c in range(3)]
    np.testing.assert_allclose(got, ref, rtol=0, atol=2e-6)


def test_fit_config_validation_messages():
    from diffrast.fit import ConfigError, FitConfig

    FitConfig().validate()
    for kw, msg in ((dict(triangles=0), "triangles must be greater than zero"),
                    (dict(sigma_end=0.0), "positive and finite"),
                    (dict(sigma_start=0.001), "greater than or equal to sigma_end"),
                    (dict(lr_color=-1.0), "learning rates must be positive")):
        with pytest.raises(ConfigError, match=msg):
            FitConfig(**kw).validate()


def test_sigma_and_seed_colors_match_the_oracle(oracle):
    from diffrast.fit import FitConfig, mean_color, seed_colors, sigma_at
    from diffrast.scenes import seed_scene_geometry

    cfg = FitConfig(iters=800)
    for i in (0, 1, 399, 798, 799):
        assert np.float32(sigma_at(cfg, i)) == np.float32(oracle.sigma_at(0.02, 0.0015, 800, i))
    tgt = np.random.default_rng(4).random((33, 41, 3)).astype(np.float32)
    p = seed_scene_geometry(40, 3)
    q = p.copy()
    seed_colors(tgt, p)
    bg = oracle.seed_colors(tgt, q)
    assert np.array_equal(p, q)
    assert mean_color(tgt) == tuple(float(x) for x in bg)


def test_cli_arguments():
    from diffrast.fit_cli import UsageError, parse_args

    assert parse_args(["--help"]) is None
    target, cfg, o = parse_args(["img.png", "--tris", "16", "--iters", "30", "--patience", "0",
                                 "--out", "d", "--quiet"])
    assert target == "img.png" and cfg.triangles == 16 and cfg.iters == 30
    assert cfg.patience is None and o["out"] == "d" and o["quiet"]
    with pytest.raises(UsageError, match="unknown option --bogus"):
        parse_args(["--bogus", "1"])
    with pytest.raises(UsageError, match="--tris requires a value"):
        parse_args(["--tris"])
    with pytest.raises(UsageError, match="--tris requires a value"):
        parse_args(["--tris", "--quiet"])
    with pytest.raises(UsageError, match="non-negative integer, got '-5'"):
        parse_args(["--iters", "-5"])
    with pytest.raises(UsageError, match="--size must be greater than zero"):
        parse_args(["--size", "0"])
    from diffrast.fit import ConfigError

    with pytest.raises(ConfigError):
        parse_args(["--tris", "0"])


def test_cli_missing_target_file_is_an_error(tmp_path):
    from diffrast.fit_cli import UsageError, run

    with pytest.raises(UsageError, match="no such file"):
        run([os.path.join(str(tmp_path), "missing.png")])
