"""The refine loop of python/evaluate.py:79-132 with the fused device Adam.

The reference refines a batch of predicted scenes by running torch's Adam over
``fused_loss``. It reads the loss back to the host every step for its PSNR
trace. Here each step is one fused forward + MSE + backward kernel and one
fused Adam kernel with projection (``dr_adam_step``, the same ranges as
``clamp_params``). The per-step mean MSE stays on the device until the end,
so the loop never waits on the host.
"""

from __future__ import annotations

import math

import torch

from . import _native


def mse_to_psnr(mse: float, max_value: float = 1.0) -> float:
    """evaluate.py:73-77."""
    if mse <= 0:
        return float("inf")
    return 10.0 * math.log10(max_value**2 / mse)


def refine(params: torch.Tensor, targets: torch.Tensor, steps: int, sigma: float,
           lr: float = 0.02) -> tuple[torch.Tensor, list[float]]:
    """Refine (B, T, 10) ``params`` towards (B, 3, H, W) ``targets``.

    Same contract as evaluate.py's ``refine``: ``trace[i]`` is the PSNR after
    exactly ``i`` steps (``steps + 1`` entries), and the gradient is that of the
    batch-mean MSE (``fused_loss`` differentiates the sum of per-item MSE, so
    it is divided by the batch size). Adam uses betas (0.9, 0.999) and eps 1e-8,
    torch's defaults. The projection also maps NaN parameters to 0.5 as
    fit.rs's ``project`` does, where ``clamp_params`` would keep NaN.
    """
    if steps < 0:
        raise ValueError("steps must be non-negative")
    dev = _native._resolve_device(params.device if params.is_cuda else None)
    p = params.detach().to(dev, torch.float32).contiguous().clone()
    hwc = targets.detach().to(dev, torch.float32).permute(0, 2, 3, 1).contiguous()
    batch = p.shape[0]
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    means = torch.empty(steps + 1, dtype=torch.float32, device=dev)
    for i in range(steps):
        losses, grads = _native.loss_backward(p, hwc, sigma)
        means[i] = losses.mean()
        grads.div_(batch)
        _native.adam_step(p, m, v, grads, i + 1, lr, lr, lr, project=True)
    losses, _ = _native.loss_backward(p, hwc, sigma)
    means[steps] = losses.mean()
    trace = [mse_to_psnr(x) for x in means.tolist()]
    return p.to(params.device), trace
