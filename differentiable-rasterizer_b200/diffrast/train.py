"""The training step's rasterizer calls on device tensors (python/train.py:127-179).

``train_step`` keeps the reference's signature and metrics: an optional
parameter-supervision term (smooth L1 against target parameters), plus the
photometric term ``fused_mse`` on the first ``render_fraction`` of the batch,
with PSNR derived from that loss. Here ``fused_mse`` runs on the model's CUDA
tensors through the fused loss + backward kernel, so neither the predicted
parameters nor the images leave the device (the reference copied both to host
numpy on every step, torch_layer.py:123-124).

``global_fused_mse`` is the data-parallel form for per-scene parameters (the
benchmark's config 3 sharded over ranks): each rank holds B_local of the B_global
scenes, so its loss is its scenes' summed MSE over B_global. The gradient each
rank gets for its own scenes is then the gradient of the single-device B_global
mean, not B_global / B_local times it. A model trained under DDP needs no such
scaling (DDP averages the ranks' gradients), and ``train_step`` does none.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor

from .torch_layer import fused_mse


def global_fused_mse(params: Tensor, targets: Tensor, global_batch: int, sigma: float = 0.0015,
                     background=(0.0, 0.0, 0.0)) -> Tensor:
    """This rank's share of the global-batch mean MSE: mean over its B_local
    scenes times B_local / B_global. Summed over ranks it is the mean over all
    B_global scenes, and its gradient on this rank's scenes is that mean's."""
    if global_batch <= 0 or params.shape[0] > global_batch:
        raise ValueError(f"global_batch {global_batch} for {params.shape[0]} local scenes")
    local = fused_mse(params, targets, sigma, background)
    return local * (params.shape[0] / global_batch)


def train_step(model, batch, args, sigma: float, device: torch.device):
    """One optimization step's loss and metrics (train.py:127-179). ``args``
    needs ``param_weight``, ``render_weight`` and ``render_fraction``; its
    ``raster_device`` is accepted and ignored (the kernels always run on CUDA)."""
    supervised = isinstance(batch, (list, tuple))
    if supervised:
        images, target_params = batch
        images = images.to(device, non_blocking=True)
        target_params = target_params.to(device, non_blocking=True)
    else:
        images = batch.to(device, non_blocking=True)
        target_params = None

    predicted = model(images)
    metrics: dict[str, float] = {}
    loss = torch.zeros((), device=device)
    if target_params is not None:
        param_loss = F.smooth_l1_loss(predicted, target_params)
        loss = loss + args.param_weight * param_loss
        metrics["param_loss"] = param_loss.item()
    if args.render_weight > 0:
        n = max(1, int(len(images) * args.render_fraction))
        render_loss = fused_mse(predicted[:n], images[:n], sigma=sigma)
        loss = loss + args.render_weight * render_loss
        metrics["render_loss"] = render_loss.item()
        mse = metrics["render_loss"]
        metrics["psnr"] = float("inf") if mse <= 0 else 10.0 * math.log10(1.0 / mse)
    metrics["loss"] = loss.item()
    return loss, metrics
