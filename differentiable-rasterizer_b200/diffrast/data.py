"""Synthetic training scenes rendered on the GPU (python/diffrast/data.py:77-126).

``SyntheticShapeDataset`` keeps the reference dataset's contract: item ``i`` is
deterministic in ``(seed, i)`` alone (a CPU ``torch.Generator`` seeded with
``seed * 1_000_003 + i`` draws ``random_params(1, triangles)`` and then a
background ``rand(3) * 0.3``), rendered at ``sigma``. The draws stay on the host,
where the reference makes them, so the parameters are bit-identical to the
reference's; the rendering runs on the device. ``batch(indices)`` renders a
whole batch in one launch (one background per scene) and returns ``(B, 3, H,
W)`` device tensors, so a training loop never round-trips images through host
memory the way ``rasterize`` on CPU tensors made the reference's loader do
(torch_layer.py:46).
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _native
from .torch_layer import random_params


class SyntheticShapeDataset(torch.utils.data.Dataset):
    """Random triangle scenes rendered on demand, on ``device``."""

    def __init__(self, length: int = 10_000, size: int = 64, triangles: int = 32,
                 sigma: float = 0.004, seed: int = 0, size_value=None,
                 device: torch.device | str = "cuda") -> None:
        self.length = length
        self.size = size
        self.triangles = triangles
        self.sigma = sigma
        self.seed = seed
        # A multiprocessing.Value shared with loader workers, as the reference
        # uses it for per-epoch resolution changes (data.py:100-106).
        self.size_value = size_value
        self.device = torch.device(device)

    def __len__(self) -> int:
        return self.length

    def _size(self) -> int:
        return self.size_value.value if self.size_value is not None else self.size

    def scene(self, index: int) -> tuple[Tensor, Tensor]:
        """Item ``index``'s parameters (1, T, 10) and background (3,), drawn as
        the reference draws them (data.py:111-115)."""
        if not 0 <= index < self.length:
            raise IndexError(index)
        gen = torch.Generator().manual_seed(self.seed * 1_000_003 + index)
        params = random_params(1, self.triangles, generator=gen)
        background = torch.rand(3, generator=gen) * 0.3
        return params, background

    def batch(self, indices) -> Tensor:
        """Images of ``indices`` as one (B, 3, H, W) tensor on the device, from
        one render launch."""
        idx = [int(i) for i in indices]
        size = self._size()
        if not idx:
            return torch.empty((0, 3, size, size), device=self.device)
        drawn = [self.scene(i) for i in idx]
        params = torch.cat([p for p, _ in drawn]).to(self.device, non_blocking=True)
        bgs = torch.stack([b for _, b in drawn])  # host: (B, 3) read by the launch
        with torch.no_grad():
            return _native.render(params, size, size, self.sigma, bgs,
                                  layout=_native.LAYOUT_BCHW)

    def __getitem__(self, index: int) -> Tensor:
        return self.batch([index])[0]


class DeviceBatches:
    """Batches of a SyntheticShapeDataset rendered straight into device memory,
    in index order (or a seeded permutation), ``batch_size`` scenes per launch."""

    def __init__(self, dataset: SyntheticShapeDataset, batch_size: int, shuffle: bool = False,
                 seed: int = 0, rank: int = 0, world_size: int = 1):
        self.ds = dataset
        self.batch_size = batch_size
        self.shuffle = shuffle
        self.seed = seed
        self.rank = rank
        self.world = world_size
        self.epoch = 0

    def set_epoch(self, epoch: int) -> None:
        self.epoch = epoch

    def __iter__(self):
        n = len(self.ds)
        if self.shuffle:
            g = torch.Generator().manual_seed(self.seed + self.epoch)
            order = torch.randperm(n, generator=g).tolist()
        else:
            order = list(range(n))
        order = order[self.rank::self.world]  # each rank its own disjoint share
        for i in range(0, len(order), self.batch_size):
            yield self.ds.batch(order[i:i + self.batch_size])

    def __len__(self) -> int:
        per_rank = (len(self.ds) - self.rank + self.world - 1) // self.world
        return (per_rank + self.batch_size - 1) // self.batch_size
