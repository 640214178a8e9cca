"""File formats of the fit artefacts, written as the reference writes them.

- ``scene_to_json``: the scene JSON of crates/diffrast/src/serial.rs:21-75
  (``{:.6}`` numbers, non-finite values written as ``0.0``, no trailing commas).
- ``loss_csv``: ``iter,loss`` rows as bin/fit.rs:196-204 writes them, each loss
  in Rust's ``f32`` Display form (shortest round-trip digits, never an exponent).
- ``encode_srgb`` / ``decode_srgb``: canvas.rs:103-120 in f32 arithmetic.
- ``write_png`` / ``read_png``: 8-bit RGB PNG files. The pixel bytes equal the
  reference's (``encode_srgb`` of the linear canvas); the compressed stream
  is zlib's, so the files are pixel-identical rather than byte-identical to
  those of the ``image`` crate.
- ``fit_within``, ``scale_to``, ``resize_lanczos3``: target preparation
  (canvas.rs:89-96, bin/fit.rs:190-194, the ``image`` crate's Lanczos3 resize as
  a separable windowed sinc of radius 3; the ``image`` crate is a third-party
  dependency, so the resize agrees to rounding, not bit for bit).
- ``synthetic_target``: the CLI's built-in target (bin/fit.rs:219-250).

Host-side code: none of it is on the rasterizer's hot path.
"""

from __future__ import annotations

import math
import struct
import zlib

import numpy as np

F32 = np.float32


# --- scene JSON (serial.rs) ---------------------------------------------------


def _fmt_f32(v) -> str:
    """serial.rs:66-72: ``{:.6}`` of the f32 value; non-finite becomes ``0.0``."""
    v = F32(v)
    if not np.isfinite(v):
        return "0.0"
    return f"{float(v):.6f}"


def _array(vals) -> str:
    return "[" + ", ".join(_fmt_f32(v) for v in vals) + "]"


def scene_to_json(params, background) -> str:
    """Scene JSON of (T, 10) parameters and an RGB background (serial.rs:21-49)."""
    p = np.asarray(params, dtype=np.float32).reshape(-1, 10)
    out = ['{\n  "version": 1,\n  "background": ', _array(background), ',\n  "triangles": [\n']
    for i, t in enumerate(p):
        verts = ", ".join(_array(t[2 * j:2 * j + 2]) for j in range(3))
        out.append(f'    {{"verts": [{verts}], "color": {_array(t[6:9])}, '
                   f'"alpha": {_fmt_f32(t[9])}}}')
        if i + 1 < len(p):
            out.append(",")
        out.append("\n")
    out.append("  ]\n}\n")
    return "".join(out)


# --- loss CSV (bin/fit.rs) ---------------------------------------------------------


def rust_f32_display(v) -> str:
    """Rust's ``Display`` for f32: the shortest digits that round-trip, in
    positional notation; ``NaN``, ``inf``, ``-inf`` as Rust spells them."""
    v = F32(v)
    if np.isnan(v):
        return "NaN"
    if np.isinf(v):
        return "inf" if v > 0 else "-inf"
    return np.format_float_positional(v, unique=True, trim="-")


def loss_csv(losses) -> str:
    """``iter,loss`` then one row per iteration (bin/fit.rs:196-204)."""
    rows = ["iter,loss\n"]
    rows += [f"{i},{rust_f32_display(l)}\n" for i, l in enumerate(np.asarray(losses, np.float32))]
    return "".join(rows)


# --- sRGB (canvas.rs) ---------------------------------------------------------------


def encode_srgb(linear) -> np.ndarray:
    """canvas.rs:103-108 in f32: clamp, the sRGB curve, ``(s * 255 + 0.5) as u8``
    (a saturating cast: NaN becomes 0)."""
    v = np.asarray(linear, dtype=np.float32)
    with np.errstate(invalid="ignore"):
        v = np.where(v < F32(0.0), F32(0.0), v)
        v = np.where(v > F32(1.0), F32(1.0), v)
        lo = F32(12.92) * v
        hi = F32(1.055) * np.power(v, F32(1.0) / F32(2.4), dtype=np.float32) - F32(0.055)
        s = np.where(v <= F32(0.0031308), lo, hi).astype(np.float32)
        x = s * F32(255.0) + F32(0.5)
    x = np.where(np.isnan(x), F32(0.0), x)
    return np.clip(np.trunc(x), 0, 255).astype(np.uint8)


def decode_srgb(u8) -> np.ndarray:
    """canvas.rs:111-118 in f32."""
    v = np.asarray(u8, dtype=np.float32) / F32(255.0)
    lo = v / F32(12.92)
    hi = np.power((v + F32(0.055)) / F32(1.055), F32(2.4), dtype=np.float32)
    return np.where(v <= F32(0.04045), lo, hi).astype(np.float32)


# --- PNG ------------------------------------------------------------------------------


def _chunk(kind: bytes, data: bytes) -> bytes:
    return (struct.pack(">I", len(data)) + kind + data +
            struct.pack(">I", zlib.crc32(kind + data) & 0xFFFFFFFF))


def png_bytes(rgb8) -> bytes:
    """An 8-bit RGB PNG of an (H, W, 3) uint8 array (filter 0 on every row)."""
    a = np.ascontiguousarray(rgb8, dtype=np.uint8)
    if a.ndim != 3 or a.shape[2] != 3:
        raise ValueError("expected an (H, W, 3) uint8 image")
    h, w = a.shape[:2]
    raw = b"".join(b"\x00" + a[y].tobytes() for y in range(h))
    ihdr = struct.pack(">IIBBBBB", w, h, 8, 2, 0, 0, 0)
    return (b"\x89PNG\r\n\x1a\n" + _chunk(b"IHDR", ihdr) + _chunk(b"IDAT", zlib.compress(raw, 6)) +
            _chunk(b"IEND", b""))


def write_png(path, linear) -> None:
    """Canvas::save_png (canvas.rs:61-68): sRGB-encode a linear (H, W, 3) image."""
    with open(path, "wb") as f:
        f.write(png_bytes(encode_srgb(linear)))


def _paeth(a, b, c):
    p = a + b - c
    pa, pb, pc = np.abs(p - a), np.abs(p - b), np.abs(p - c)
    return np.where((pa <= pb) & (pa <= pc), a, np.where(pb <= pc, b, c))


def read_png(path) -> np.ndarray:
    """An 8-bit, non-interlaced PNG (grey, grey+alpha, RGB or RGBA) as (H, W, 3)
    uint8; alpha is dropped as the ``image`` crate's ``to_rgb8`` drops it."""
    with open(path, "rb") as f:
        data = f.read()
    if data[:8] != b"\x89PNG\r\n\x1a\n":
        raise ValueError(f"{path}: not a PNG file")
    pos, idat, ihdr = 8, [], None
    while pos < len(data):
        (n,) = struct.unpack(">I", data[pos:pos + 4])
        kind = data[pos + 4:pos + 8]
        body = data[pos + 8:pos + 8 + n]
        pos += 12 + n
        if kind == b"IHDR":
            ihdr = struct.unpack(">IIBBBBB", body)
        elif kind == b"IDAT":
            idat.append(body)
        elif kind == b"IEND":
            break
    if ihdr is None:
        raise ValueError(f"{path}: no IHDR chunk")
    w, h, depth, ctype, _, _, interlace = ihdr
    channels = {0: 1, 2: 3, 4: 2, 6: 4}.get(ctype)
    if depth != 8 or channels is None or interlace != 0:
        raise ValueError(f"{path}: only 8-bit non-interlaced grey/RGB(A) PNGs are supported")
    raw = np.frombuffer(zlib.decompress(b"".join(idat)), dtype=np.uint8)
    stride = w * channels
    raw = raw[:h * (stride + 1)].reshape(h, stride + 1)
    out = np.zeros((h, stride), dtype=np.int32)
    prev = np.zeros(stride, dtype=np.int32)
    for y in range(h):
        ft, line = raw[y, 0], raw[y, 1:].astype(np.int32)
        if ft == 0:
            cur = line
        elif ft == 2:
            cur = (line + prev) & 0xFF
        else:
            cur = np.zeros(stride, dtype=np.int32)
            for x in range(stride):
                left = cur[x - channels] if x >= channels else 0
                up = prev[x]
                ul = prev[x - channels] if x >= channels else 0
                if ft == 1:
                    pred = left
                elif ft == 3:
                    pred = (left + up) >> 1
                elif ft == 4:
                    pred = int(_paeth(np.int32(left), np.int32(up), np.int32(ul)))
                else:
                    raise ValueError(f"{path}: bad filter type {ft}")
                cur[x] = (line[x] + pred) & 0xFF
        out[y] = cur
        prev = cur
    img = out.reshape(h, w, channels).astype(np.uint8)
    if channels in (1, 2):
        img = np.repeat(img[..., :1], 3, axis=2)
    return np.ascontiguousarray(img[..., :3])


# --- target preparation ---------------------------------------------------------------


def fit_within(w: int, h: int, max_side: int) -> tuple[int, int]:
    """canvas.rs:89-96: scale down (never up) so neither side exceeds max_side."""
    if max_side == 0 or w == 0 or h == 0 or (w <= max_side and h <= max_side):
        return max(w, 1), max(h, 1)
    scale = max_side / max(w, h)
    return max(int(round_half_away(w * scale)), 1), max(int(round_half_away(h * scale)), 1)


def scale_to(w: int, h: int, target: int) -> tuple[int, int]:
    """bin/fit.rs:190-194: scale so the longest side is `target`, either way."""
    scale = target / max(w, h)
    return max(int(round_half_away(w * scale)), 1), max(int(round_half_away(h * scale)), 1)


def round_half_away(x: float) -> float:
    """Rust's f64::round: halves away from zero."""
    return math.floor(x + 0.5) if x >= 0 else -math.floor(-x + 0.5)


def _lanczos3(x):
    x = np.asarray(x, dtype=np.float64)
    out = np.sinc(x) * np.sinc(x / 3.0)
    return np.where(np.abs(x) < 3.0, out, 0.0)


def _resample_axis(a: np.ndarray, n_out: int, axis: int) -> np.ndarray:
    n_in = a.shape[axis]
    scale = n_in / n_out
    support = 3.0 * max(scale, 1.0)
    filt = max(scale, 1.0)
    centres = (np.arange(n_out) + 0.5) * scale
    lo = np.floor(centres - support).astype(int)
    taps = int(math.ceil(2 * support)) + 1
    idx = lo[:, None] + np.arange(taps)[None, :]
    w = _lanczos3((idx + 0.5 - centres[:, None]) / filt)
    valid = (idx >= 0) & (idx < n_in)
    w = np.where(valid, w, 0.0)
    w /= np.maximum(w.sum(axis=1, keepdims=True), 1e-12)
    idx = np.clip(idx, 0, n_in - 1)
    moved = np.moveaxis(a, axis, 0)
    res = np.einsum("ot,ot...->o...", w, moved[idx])
    return np.moveaxis(res, 0, axis)


def resize_lanczos3(rgb8, width: int, height: int) -> np.ndarray:
    """Resize an (H, W, 3) uint8 image with a separable Lanczos3 filter (widened
    by the scale factor when shrinking), rounding and clamping to uint8."""
    a = np.asarray(rgb8, dtype=np.float64)
    a = _resample_axis(a, width, axis=1)
    a = _resample_axis(a, height, axis=0)
    return np.clip(np.floor(a + 0.5), 0, 255).astype(np.uint8)


def load_target(path, max_side: int) -> np.ndarray:
    """bin/fit.rs:176-188 + Canvas::load_image: a PNG resized to fit within
    max_side (aspect kept), decoded to linear (H, W, 3) f32."""
    img = read_png(path)
    h, w = img.shape[:2]
    tw, th = fit_within(w, h, max_side)
    if (tw, th) != (w, h):
        img = resize_lanczos3(img, tw, th)
    return decode_srgb(img)


def _coverage(verts, px, py, sigma):
    """raster.rs:74-106 in numpy f32: sigmoid(signed distance / sigma)."""
    v = np.asarray(verts, dtype=np.float32).reshape(3, 2)
    d = np.full(px.shape, np.inf, dtype=np.float32)
    crosses = []
    for i in range(3):
        ax, ay = v[i]
        bx, by = v[(i + 1) % 3]
        abx, aby = F32(bx - ax), F32(by - ay)
        apx, apy = px - ax, py - ay
        len2 = F32(abx * abx + aby * aby)
        if len2 <= F32(1e-20):
            t = np.zeros_like(px)
        else:
            t = np.clip((apx * abx + apy * aby) / len2, F32(0.0), F32(1.0))
        dx, dy = apx - t * abx, apy - t * aby
        d = np.minimum(d, np.sqrt(dx * dx + dy * dy))
        crosses.append(abx * apy - aby * apx)
    c0, c1, c2 = crosses
    inside = ((c0 >= 0) & (c1 >= 0) & (c2 >= 0)) | ((c0 <= 0) & (c1 <= 0) & (c2 <= 0))
    x = np.where(inside, d, -d) / F32(max(sigma, 1e-8))
    with np.errstate(over="ignore"):
        e = np.exp(-np.abs(x))
        return np.where(x >= 0, F32(1.0) / (F32(1.0) + e), e / (F32(1.0) + e)).astype(np.float32)


def synthetic_target(size: int) -> np.ndarray:
    """bin/fit.rs:219-250: a colour gradient plus two hard-edged opaque
    triangles composited where coverage exceeds 1e-4. (H, W, 3) f32 linear."""
    i = np.arange(size, dtype=np.float32)
    u = (i / F32(size))[None, :]
    v = (i / F32(size))[:, None]
    c = np.empty((size, size, 3), dtype=np.float32)
    c[..., 0] = F32(0.15) + F32(0.5) * u
    c[..., 1] = F32(0.10) + F32(0.4) * v
    c[..., 2] = F32(0.55) - F32(0.3) * u
    shapes = [([[0.15, 0.70], [0.55, 0.68], [0.35, 0.20]], [0.95, 0.85, 0.25]),
              ([[0.50, 0.30], [0.88, 0.45], [0.62, 0.85]], [0.10, 0.25, 0.45])]
    centre = (i + F32(0.5)) / F32(size)
    px, py = np.meshgrid(centre, centre)
    for verts, colour in shapes:
        w = _coverage(verts, px, py, 0.002)
        m = w > F32(1e-4)
        for ch in range(3):
            out = F32(colour[ch]) * w + c[..., ch] * (F32(1.0) - w)
            c[..., ch] = np.where(m, out, c[..., ch])
    return c
