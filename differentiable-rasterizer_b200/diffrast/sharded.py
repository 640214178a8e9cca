"""One large scene split across GPUs: by tile rows (benchmark config 4,
``ShardedSceneStep``) or by triangle blocks (``TriangleShardedStep``).

Each rank renders and differentiates only the 16-pixel tile rows
``r % world == rank`` (``dr_loss_backward_sharded``): image rows are disjoint,
so the forward needs no communication. The ranks then all-reduce one buffer
holding the partial T x 10 gradient and the partial f64 sum of squared error,
and every rank applies the same Adam step, so the parameters stay identical
without a broadcast. The reference has no multi-device path; the sum over
shards equals the single-device ``dr_loss_backward`` (tested).

One process per GPU, ``torch.distributed`` with the NCCL backend for the
all-reduce (gloo works too, for CPU-side tests of the plumbing).
"""

from __future__ import annotations

import torch

from . import _native

TILE = 16


def shard_rows(height: int, shard: int, n_shards: int) -> list[int]:
    """Tile rows a shard covers: every n-th 16-pixel row, interleaved so that
    bands of dense geometry spread over all ranks."""
    if not (0 <= shard < n_shards):
        raise ValueError(f"shard {shard} of {n_shards}")
    tiles_y = (height + TILE - 1) // TILE
    return list(range(shard, tiles_y, n_shards))


class ShardedSceneStep:
    """Forward + MSE + backward of one (or a few) large scenes across ranks, then
    Adam with the fit's per-parameter rates and projection (fit.rs:388-424)."""

    def __init__(self, params: torch.Tensor, group=None, lr_pos=0.004, lr_color=0.02,
                 lr_alpha=0.01):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if params.dim() != 3 or params.shape[-1] != _native.N_PARAMS:
            raise ValueError("params must be (B, T, 10)")
        self.params = params.detach().to(torch.float32).contiguous()
        self.m = torch.zeros_like(self.params)
        self.v = torch.zeros_like(self.params)
        self.t = 0
        self.lrs = (lr_pos, lr_color, lr_alpha)
        # The kernel writes this rank's partial gradient and f64 loss sums
        # straight into these buffers, which the all-reduces then sum in place:
        # no copies or conversions between the kernel and Adam.
        self.grads = torch.empty_like(self.params)
        self.sums = torch.empty(self.params.shape[0], dtype=torch.float64,
                                device=self.params.device)

    def loss_and_grads(self, targets: torch.Tensor, sigma: float, background=(0.0, 0.0, 0.0)):
        """All-reduced (losses (B,), grads (B, T, 10)) for the current params.
        The returned gradient is the step's buffer: the next call overwrites it."""
        _native.loss_backward_sharded(self.params, targets, sigma, self.rank, self.world,
                                      background, out=(self.grads, self.sums))
        if self.world > 1:
            self.dist.all_reduce(self.grads, op=self.dist.ReduceOp.SUM, group=self.group)
            self.dist.all_reduce(self.sums, op=self.dist.ReduceOp.SUM, group=self.group)
        h, w = targets.shape[1], targets.shape[2]
        losses = (self.sums / float(h * w * 3)).to(torch.float32)  # canvas.rs:58
        return losses, self.grads

    def step(self, targets: torch.Tensor, sigma: float, background=(0.0, 0.0, 0.0)):
        """One fit iteration: loss, gradients, Adam + projection. Returns losses."""
        losses, grads = self.loss_and_grads(targets, sigma, background)
        self.t += 1
        _native.adam_step(self.params, self.m, self.v, grads, self.t, *self.lrs)
        return losses


def triangle_block(T: int, n_blocks: int, block: int) -> tuple[int, int]:
    """Triangles [t0, t1) of block `block` of `n_blocks` (ceil(T / n) each, the
    last one shorter or empty), as dr_triangle_block_* cut them."""
    if not (0 <= block < n_blocks):
        raise ValueError(f"block {block} of {n_blocks}")
    per = -(-T // n_blocks)
    t0 = min(T, block * per)
    return t0, min(T, t0 + per)


class TriangleShardedStep:
    """One scene batch sharded by triangle blocks: rank r owns the triangles of
    block r (``triangle_block``). This is the compositing-chain split of a
    single scene across GPUs, for scenes whose triangle count, not pixel count,
    is the problem.

    Per step:
    1. ``dr_triangle_block_forward`` runs the rank's block over every pixel;
    2. one all-gather exchanges the blocks' per-pixel states (32 bytes per pixel
       and block);
    3. ``dr_triangle_block_backward`` combines the blocks (the same image and
       loss on every rank) and runs the gradient pass of the rank's own block;
    4. Adam updates the parameters, and only the own block moves: the others get
       zero gradient, keep zero moments and stay put.

    No gradient or parameter exchange is needed, since a rank only renders its
    own block. ``gather_params`` assembles the full parameters when wanted.
    """

    def __init__(self, params: torch.Tensor, group=None, lr_pos=0.004, lr_color=0.02,
                 lr_alpha=0.01):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if params.dim() != 3 or params.shape[-1] != _native.N_PARAMS:
            raise ValueError("params must be (B, T, 10)")
        self.params = params.detach().to(torch.float32).contiguous()
        self.m = torch.zeros_like(self.params)
        self.v = torch.zeros_like(self.params)
        self.t = 0
        self.lrs = (lr_pos, lr_color, lr_alpha)
        self.t0, self.t1 = triangle_block(self.params.shape[1], self.world, self.rank)

    def loss_and_grads(self, targets: torch.Tensor, sigma: float, background=(0.0, 0.0, 0.0)):
        """(losses (B,), grads (B, T, 10) nonzero on this rank's block)."""
        h, w = targets.shape[1], targets.shape[2]
        state = _native.triangle_block_state(self.params, h, w, self.world)
        _native.triangle_block_forward(self.params, h, w, sigma, self.world, self.rank, state,
                                       background)
        if self.world > 1:
            own = state[self.rank].reshape(-1).clone()
            self.dist.all_gather_into_tensor(state.view(-1), own, group=self.group)
        return _native.triangle_block_backward(self.params, state, targets, sigma, self.world,
                                               self.rank, background)

    def step(self, targets: torch.Tensor, sigma: float, background=(0.0, 0.0, 0.0)):
        """One fit iteration: loss, gradients, Adam + projection. Returns losses."""
        losses, grads = self.loss_and_grads(targets, sigma, background)
        self.t += 1
        _native.adam_step(self.params, self.m, self.v, grads, self.t, *self.lrs)
        return losses

    def gather_params(self) -> torch.Tensor:
        """The full (B, T, 10) parameters, each block from its owner."""
        if self.world == 1:
            return self.params.clone()
        full = torch.zeros_like(self.params)
        full[:, self.t0:self.t1] = self.params[:, self.t0:self.t1]
        self.dist.all_reduce(full, op=self.dist.ReduceOp.SUM, group=self.group)
        return full
