"""The rasterizer as a PyTorch operation, on B200 kernels.

Drop-in for the reference's ``python/diffrast/torch_layer.py`` (same names,
signatures, argument meaning and errors). The difference is underneath: the
reference copies every tensor to CPU numpy and calls a Rust/wgpu extension
(torch_layer.py:42-47); here CUDA tensors stay on the device and the
``libdiffrast_cuda.so`` kernels read and write them in place on the current
stream. CPU tensors are accepted too: they are copied to the current CUDA
device, and results come back on the tensor's own device, as the reference
returns them (torch_layer.py:107).

    params = model(image)                    # (B, T, 10)
    render = rasterize(params, 128, 128)     # (B, 3, H, W)
    loss = F.mse_loss(render, image)
    loss.backward()                          # gradients reach `model`

There is no CPU path: ``device="cpu"`` raises, and so does any call when the
library or a CUDA device is missing.
"""

from __future__ import annotations

import atexit

import torch
from torch import Tensor

from . import _native

#: Parameters per triangle: 6 position + 3 color + 1 alpha.
N_PARAMS: int = _native.N_PARAMS

_last_device = "gpu"


def _parse_device(device: str) -> None:
    """diffrast-py/src/lib.rs:85-94 accepts "cpu", "gpu", "cuda", "auto"."""
    if device in ("gpu", "cuda", "auto"):
        return
    if device == "cpu":
        raise ValueError(
            'device="cpu": this build has no CPU rasterizer; it runs only on CUDA '
            '(use "gpu", "cuda" or "auto")')
    raise ValueError(f'unknown device {device!r} — expected "cpu", "gpu" or "auto"')


def _note_gpu() -> None:
    global _last_device
    _last_device = "gpu"


def _check_params(params: Tensor) -> None:
    if params.dim() != 3 or params.shape[-1] != N_PARAMS:
        raise ValueError(
            f"expected params of shape (B, T, {N_PARAMS}), got {tuple(params.shape)}")


def _check_sigma(sigma: float) -> None:
    if not (sigma > 0):
        raise ValueError("sigma must be positive")


# Largest pixel tape (16 bytes per pixel of the batch) the forward keeps for
# the backward; larger batches recompute the forward in the backward.
_TAPE_LIMIT = 1 << 29


class _Rasterize(torch.autograd.Function):
    """Forward = dr_render_taped (the image, plus each pixel's running product
    of 1 - w); backward = dr_grad_backward_taped on the upstream gradient,
    which reads the products back instead of running the forward walk again
    (BackwardMode::Taped, compact). Calls that need no parameter gradient, and
    batches whose tape would exceed _TAPE_LIMIT, take dr_render /
    dr_grad_backward."""

    @staticmethod
    def forward(ctx, params: Tensor, height: int, width: int, sigma: float, background,
                channels_first: bool):
        layout = _native.LAYOUT_BCHW if channels_first else _native.LAYOUT_BHWC
        B = params.shape[0]
        tape = None
        if ctx.needs_input_grad[0] and _native.pixel_tape_bytes(B, height, width) <= _TAPE_LIMIT:
            images, tape = _native.render_taped(params, height, width, sigma, background, layout)
        else:
            images = _native.render(params, height, width, sigma, background, layout)
        _note_gpu()
        if tape is None:
            ctx.save_for_backward(params)
        else:
            ctx.save_for_backward(params, tape)
        ctx.sigma = sigma
        ctx.background = background
        ctx.layout = layout
        return images

    @staticmethod
    def backward(ctx, grad_images: Tensor):
        saved = ctx.saved_tensors
        params = saved[0]
        if len(saved) == 2:
            grads = _native.grad_backward_taped(params, grad_images, saved[1], ctx.sigma,
                                                ctx.background, ctx.layout)
        else:
            grads = _native.grad_backward(params, grad_images, ctx.sigma, ctx.background,
                                          ctx.layout)
        _note_gpu()
        grad_params = grads.to(params.device, params.dtype)
        return grad_params, None, None, None, None, None


def rasterize(
    params: Tensor,
    height: int,
    width: int,
    sigma: float = 0.0015,
    background: tuple[float, float, float] = (0.0, 0.0, 0.0),
    channels_first: bool = True,
    device: str = "auto",
) -> Tensor:
    """Differentiable batched render (same signature as torch_layer.py:69-108).

    Args:
        params: ``(B, T, 10)`` float tensor. Each row holds one triangle's three
            vertices ``x0, y0, x1, y1, x2, y2`` (the unit square maps onto the
            image), its colour ``r, g, b`` and its opacity ``a``; row 0 is
            painted first, so later rows cover earlier ones.
        height, width: image size in pixels.
        sigma: width of the soft edge, as a fraction of the image side: the
            coverage of a pixel falls from 1 to 0 over a few ``sigma`` around
            each edge.
        background: the RGB value every pixel starts from before any triangle
            is painted.
        channels_first: ``(B, 3, H, W)`` when true (the kernel writes that
            layout directly), ``(B, H, W, 3)`` when false.
        device: ``"auto"``, ``"gpu"`` or ``"cuda"``; every choice runs the
            CUDA kernels (there is no CPU path).

    Returns:
        The images, linear RGB values, on ``params.device``.
    """
    _check_params(params)
    if height <= 0 or width <= 0:
        raise ValueError("height and width must be positive")
    _check_sigma(sigma)
    _parse_device(device)
    images = _Rasterize.apply(params, height, width, sigma, background, channels_first)
    return images.to(params.device, params.dtype)


class _FusedMSE(torch.autograd.Function):
    """Photometric MSE against a target in one kernel (torch_layer.py:111-138)."""

    @staticmethod
    def forward(ctx, params: Tensor, targets: Tensor, sigma: float, background):
        losses, grads = _native.loss_backward(params, targets, sigma, background,
                                              _native.LAYOUT_BCHW)
        _note_gpu()
        ctx.save_for_backward(grads.to(params.device, params.dtype))
        ctx.batch = len(params)
        return losses.mean().to(params.device, params.dtype)

    @staticmethod
    def backward(ctx, grad_out: Tensor):
        (grads,) = ctx.saved_tensors
        # The kernel differentiates the *sum* of per-item MSE; the forward
        # returns their mean, so the chain rule needs the 1/B.
        return grad_out * grads / ctx.batch, None, None, None


def fused_mse(
    params: Tensor,
    targets: Tensor,
    sigma: float = 0.0015,
    background: tuple[float, float, float] = (0.0, 0.0, 0.0),
    device: str = "auto",
) -> Tensor:
    """``F.mse_loss(rasterize(params, H, W, sigma), targets)`` with one render.

    Args:
        params: ``(B, T, 10)`` scene parameters.
        targets: ``(B, 3, H, W)``, matching what ``rasterize`` returns. Read in
            place in that layout (no permute copy).
    """
    _check_params(params)
    if targets.dim() != 4 or targets.shape[1] != 3:
        raise ValueError(f"expected targets of shape (B, 3, H, W), got {tuple(targets.shape)}")
    _check_sigma(sigma)
    _parse_device(device)
    if targets.shape[0] != params.shape[0]:
        raise ValueError(
            f"batch mismatch: {params.shape[0]} parameter rows but {targets.shape[0]} targets")
    return _FusedMSE.apply(params, targets, sigma, background)


def gpu_adapter() -> str | None:
    """Name of the CUDA device the kernels run on, or ``None`` without one."""
    try:
        if _native.device_count() == 0:
            return None
        return _native.device_name(torch.cuda.current_device() if torch.cuda.is_available() else 0)
    except ImportError:
        return None


def last_device() -> str:
    """Device the most recent call ran on: always ``"gpu"`` in this build."""
    return _last_device


def shutdown_gpu() -> bool:
    """Release the library's CUDA contexts (scratch memory) now."""
    return _native.shutdown()


atexit.register(shutdown_gpu)


def policy_prefers_gpu(batch: int, triangles: int, pixels: int,
                       discrete: bool | None = None) -> bool:
    """The reference's ``device="auto"`` size rule (diffrast-py/src/lib.rs:138-147).

    Kept for API compatibility. This build has no CPU path, so ``auto`` always
    runs the CUDA kernels; the rule only answers what the reference would pick.
    """
    if discrete is None:
        discrete = True
    if not discrete:
        return batch >= 4 and batch * triangles * pixels >= 1_000_000_000
    return batch >= 2 and batch * triangles * pixels >= 250_000


def fused_loss(
    params: Tensor,
    targets: Tensor,
    sigma: float = 0.0015,
    background: tuple[float, float, float] = (0.0, 0.0, 0.0),
    device: str = "auto",
) -> tuple[Tensor, Tensor]:
    """Per-item MSE and parameter gradients in one call, without autograd.

    Args:
        targets: ``(B, H, W, 3)``.

    Returns:
        ``(losses, grads)`` — ``(B,)`` and ``(B, T, 10)``, on ``params.device``.
    """
    if targets.dim() != 4:
        raise ValueError(f"expected targets of shape (B, H, W, 3), got {tuple(targets.shape)}")
    _check_params(params)
    _parse_device(device)
    if targets.shape[3] != 3:
        raise ValueError("targets must have 3 channels")
    if targets.shape[0] != params.shape[0]:
        raise ValueError(
            f"batch mismatch: {params.shape[0]} parameter rows but {targets.shape[0]} targets")
    if not (sigma > 0) or sigma == float("inf"):
        raise ValueError("sigma must be positive and finite")
    if params.device.type == "cpu" and targets.device.type == "cpu":
        # Host buffers end to end: uploads, kernels and downloads pipelined in
        # the library (dr_loss_backward_host), one call, results in host memory.
        losses, grads = _native.loss_backward_host(params, targets, sigma, background,
                                                   _native.LAYOUT_BHWC)
        _note_gpu()
        return losses, grads.to(params.dtype)
    losses, grads = _native.loss_backward(params, targets, sigma, background, _native.LAYOUT_BHWC)
    _note_gpu()
    return losses.to(params.device), grads.to(params.device, params.dtype)


def random_params(
    batch: int,
    triangles: int,
    *,
    device: torch.device | str = "cpu",
    generator: torch.Generator | None = None,
) -> Tensor:
    """Small random triangles (torch_layer.py:256-279, same draw order)."""
    centers = torch.rand(batch, triangles, 1, 2, device=device, generator=generator)
    offsets = (
        torch.rand(batch, triangles, 3, 2, device=device, generator=generator) - 0.5
    ) * 0.3
    verts = (centers + offsets).reshape(batch, triangles, 6)
    colors = torch.rand(batch, triangles, 3, device=device, generator=generator)
    alphas = torch.rand(batch, triangles, 1, device=device, generator=generator) * 0.4 + 0.3
    return torch.cat([verts, colors, alphas], dim=-1)


def clamp_params(params: Tensor) -> Tensor:
    """Project parameters back into their valid ranges (torch_layer.py:282-291)."""
    verts = params[..., :6].clamp(-0.25, 1.25)
    colors = params[..., 6:9].clamp(0.0, 1.0)
    alpha = params[..., 9:10].clamp(1e-3, 0.999)
    return torch.cat([verts, colors, alpha], dim=-1)


def psnr(a: Tensor, b: Tensor, max_value: float = 1.0) -> Tensor:
    """Peak signal-to-noise ratio in dB (torch_layer.py:294-303)."""
    mse = torch.mean((a - b) ** 2)
    if mse == 0:
        return torch.tensor(float("inf"), device=a.device)
    return 10.0 * torch.log10(max_value**2 / mse)


def activate(raw: Tensor, vertex_range: float = 0.15) -> Tensor:
    """TriangleNet.activate (python/diffrast/model.py:162-175): squash raw
    network output into valid parameters (config 3's input decoding)."""
    lo, hi = -vertex_range, 1.0 + vertex_range
    verts = torch.sigmoid(raw[..., :6]) * (hi - lo) + lo
    colors = torch.sigmoid(raw[..., 6:9])
    alpha = torch.sigmoid(raw[..., 9:10]) * 0.998 + 0.001
    return torch.cat([verts, colors, alpha], dim=-1)
