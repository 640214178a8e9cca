"""Module-compatible replacement for the reference's PyO3 extension ``diffrast_rs``.

Same functions and signatures as crates/diffrast-py/src/lib.rs:172-486, backed
by the sm_100a kernels of libdiffrast_cuda.so instead of Rust + wgpu:

- numpy ``float32`` arrays in -> numpy arrays out, as the reference (the
  arrays are copied to the GPU and the results back: the host-buffer path);
- CUDA torch tensors in -> CUDA tensors out, with no host round trip.

``device`` accepts "gpu", "cuda" and "auto"; "cpu" raises ValueError because
this build has no CPU rasterizer (there is no silent fallback either).
"""

from __future__ import annotations

import numpy as np
import torch

from diffrast import _native

__version__ = "0.1.0"

_last = "gpu"


def _device(device: str) -> None:
    if device in ("gpu", "cuda", "auto"):
        return
    if device == "cpu":
        raise ValueError('device="cpu": this build has no CPU rasterizer; use "gpu" or "auto"')
    raise ValueError(f'unknown device {device!r} — expected "cpu", "gpu" or "auto"')


def _to_tensor(x, ndim: int, what: str):
    """(tensor, came_from_numpy)."""
    if isinstance(x, torch.Tensor):
        t = x
        numpy_in = False
    else:
        t = torch.from_numpy(np.ascontiguousarray(np.asarray(x, dtype=np.float32)))
        numpy_in = True
    if t.dim() != ndim:
        raise ValueError(f"{what} must have {ndim} dimensions, got {t.dim()}")
    return t, numpy_in


def _out(t: torch.Tensor, numpy_out: bool):
    return t.cpu().numpy() if numpy_out else t


def _bg(background):
    return tuple(float(v) for v in background)


def _check_sigma(sigma: float) -> float:
    s = float(sigma)
    if not np.isfinite(s) or s <= 0.0:
        raise ValueError("sigma must be positive and finite")
    return s


def render_batch(params, height: int, width: int, sigma: float,
                 background=(0.0, 0.0, 0.0), device: str = "auto"):
    """(B, T, 10) params -> (B, H, W, 3) images (diffrast-py/src/lib.rs:172-231)."""
    global _last
    _device(device)
    sigma = _check_sigma(sigma)
    if height == 0 or width == 0:
        raise ValueError("height and width must be non-zero")
    p, np_in = _to_tensor(params, 3, "params")
    if p.shape[2] != _native.N_PARAMS:
        raise ValueError(f"expected last dimension {_native.N_PARAMS}, got {p.shape[2]}")
    img = _native.render(p, height, width, sigma, _bg(background), _native.LAYOUT_BHWC)
    _last = "gpu"
    return _out(img, np_in)


def backward_batch(params, grad_images, sigma: float, background=(0.0, 0.0, 0.0),
                   device: str = "auto"):
    """Upstream image gradients (B, H, W, 3) -> parameter gradients (B, T, 10)
    (diffrast-py/src/lib.rs:243-324)."""
    global _last
    _device(device)
    sigma = _check_sigma(sigma)
    p, np_in = _to_tensor(params, 3, "params")
    g, _ = _to_tensor(grad_images, 4, "grad_images")
    if p.shape[2] != _native.N_PARAMS:
        raise ValueError(f"expected last parameter dimension {_native.N_PARAMS}, got {p.shape[2]}")
    if g.shape[0] != p.shape[0]:
        raise ValueError(
            f"batch mismatch: {p.shape[0]} parameter rows but {g.shape[0]} gradient images")
    if g.shape[3] != 3:
        raise ValueError("gradient images must have 3 channels")
    grads = _native.grad_backward(p, g, sigma, _bg(background), _native.LAYOUT_BHWC)
    _last = "gpu"
    return _out(grads, np_in)


def fused_loss_backward(params, targets, sigma: float, background=(0.0, 0.0, 0.0),
                        device: str = "auto"):
    """Render, score against targets (B, H, W, 3) and differentiate in one call.
    Returns ``(losses: list[float], grads (B, T, 10))`` (diffrast-py/src/lib.rs:331-412)."""
    global _last
    _device(device)
    sigma = _check_sigma(sigma)
    p, np_in = _to_tensor(params, 3, "params")
    t, _ = _to_tensor(targets, 4, "targets")
    if p.shape[2] != _native.N_PARAMS:
        raise ValueError(f"expected last parameter dimension {_native.N_PARAMS}, got {p.shape[2]}")
    if t.shape[0] != p.shape[0]:
        raise ValueError(f"batch mismatch: {p.shape[0]} parameter rows but {t.shape[0]} targets")
    if t.shape[3] != 3:
        raise ValueError("targets must have 3 channels")
    losses, grads = _native.loss_backward(p, t, sigma, _bg(background), _native.LAYOUT_BHWC)
    _last = "gpu"
    return losses.cpu().tolist(), _out(grads, np_in)


def last_device() -> str:
    """Device used by the most recent call: always "gpu" in this build."""
    return _last


def shutdown_gpu() -> bool:
    """Release the library's CUDA contexts now (diffrast-py/src/lib.rs:435-444)."""
    return _native.shutdown()


def gpu_adapter():
    """Name of the CUDA device in use, or None (diffrast-py/src/lib.rs:447-450)."""
    try:
        if _native.device_count() == 0:
            return None
        return _native.device_name(torch.cuda.current_device() if torch.cuda.is_available() else 0)
    except ImportError:
        return None


def params_per_triangle() -> int:
    return _native.N_PARAMS


def policy_prefers_gpu(batch: int, tris: int, pixels: int, discrete=None) -> bool:
    """The reference's auto size rule (diffrast-py/src/lib.rs:138-147, 467-472)."""
    from diffrast.torch_layer import policy_prefers_gpu as rule
    return rule(batch, tris, pixels, discrete)
