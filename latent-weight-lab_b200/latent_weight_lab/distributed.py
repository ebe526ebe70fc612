"""Multi-GPU BlockFHT: block-sharded generation and tensor-parallel BlockFHTLinear.

The reference is single-process (it has no torch.distributed code); these
are the B200 build's multi-GPU forms of the same computations, one process
per GPU over NCCL.

* Blocks are independent and share only the read-only latent, so
  ``ShardedBlockFHT`` gives rank r a contiguous, block-aligned range of the
  generated coordinates; the forward needs no communication and the backward
  all-reduces the [L] latent-gradient partials (the only exchange).
* ``ColumnParallelBlockFHTLinear`` splits the output features: rank r's rows
  [r0, r1) of W are the contiguous flat range [r0*in, r1*in), generated with a
  slice of the generator.  Output is sharded on features (gather optional).
* ``RowParallelBlockFHTLinear`` splits the input features: every rank
  generates the whole W and keeps its columns (generation is replicated);
  partial outputs are all-reduced.

Every collective goes through torch.distributed on the default (or given)
process group; with the NCCL backend that is NVLink/NVSwitch on one node.
The compute callables default to the CUDA library; tests substitute a CPU
restatement to exercise the sharding and collective logic on gloo ranks.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from .block_fht import BlockFHT, block_fht_slice, next_power_of_two

SliceFn = Callable[[torch.Tensor, int, int, int, int, int], torch.Tensor]


def _world(group) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def block_shard(size: int, block_size: int, rank: int, world: int) -> tuple[int, int]:
    """Block-aligned coordinate range [start, stop) owned by `rank` (balanced by blocks)."""
    nblocks = (int(size) + block_size - 1) // block_size
    lo = (nblocks * rank) // world
    hi = (nblocks * (rank + 1)) // world
    return min(lo * block_size, size), min(hi * block_size, size)


def even_shard(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous range of n items for `rank` (sizes differ by at most one)."""
    return (n * rank) // world, (n * (rank + 1)) // world


class _AllReduceGrad(torch.autograd.Function):
    """Identity forward; all-reduce (sum) of the gradient in backward."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        if dist.is_initialized():
            dist.all_reduce(g, group=ctx.group)
        return g, None


class _AllReduceSum(torch.autograd.Function):
    """All-reduce (sum) in forward; identity backward (each rank keeps its gradient)."""

    @staticmethod
    def forward(ctx, x, group):
        y = x.contiguous().clone()
        if dist.is_initialized():
            dist.all_reduce(y, group=group)
        return y

    @staticmethod
    def backward(ctx, g):
        return g, None


class _GatherLastDim(torch.autograd.Function):
    """All-gather of feature shards along the last dim; backward keeps the local slice."""

    @staticmethod
    def forward(ctx, x, sizes, rank, group):
        ctx.sizes, ctx.rank = list(sizes), rank
        x = x.contiguous()
        if not dist.is_initialized():
            return x
        lead = x.shape[:-1]
        parts = [x.new_empty(*lead, s) for s in sizes]
        dist.all_gather(parts, x, group=group)
        return torch.cat(parts, dim=-1)

    @staticmethod
    def backward(ctx, g):
        lo = sum(ctx.sizes[: ctx.rank])
        return g[..., lo: lo + ctx.sizes[ctx.rank]].contiguous(), None, None, None


class ShardedBlockFHT(nn.Module):
    """A BlockFHT whose generated coordinates are split by whole blocks across ranks.

    ``forward()`` returns this rank's shard; ``shard_range`` says which
    coordinates those are.  The latent is replicated; its gradient is summed
    over ranks in backward, so every rank ends with the full gradient.
    """

    def __init__(self, generator: BlockFHT, group=None, slice_fn: SliceFn | None = None):
        super().__init__()
        self.generator = generator
        self.group = group
        self.slice_fn = slice_fn or block_fht_slice
        world, rank = _world(group)
        self.shard_range = block_shard(generator.size, generator.block_size, rank, world)

    def forward(self) -> torch.Tensor:
        start, stop = self.shard_range
        latent = _AllReduceGrad.apply(self.generator.latent, self.group)
        g = self.generator
        return self.slice_fn(latent, g.size, g.layers, g.seed, start, stop)


class ColumnParallelBlockFHTLinear(nn.Module):
    """Output-feature-split BlockFHTLinear: rank r owns W rows [r0, r1).

    The latent (and so the generator) is replicated; each rank generates only
    its contiguous flat range of W.  ``gather_output`` all-gathers the
    feature shards, otherwise the output stays sharded (feed it to a
    RowParallelBlockFHTLinear, Megatron style).
    """

    def __init__(self, in_features: int, out_features: int, latent_dim: int, layers: int = 3, seed: int = 0,
                 weight_scale: float = 1.0, bias: bool = False, gather_output: bool = False,
                 latent_init_std: float = 0.02, group=None, slice_fn: SliceFn | None = None):
        super().__init__()
        self.in_features, self.out_features = int(in_features), int(out_features)
        self.generator = BlockFHT(int(latent_dim), size=self.in_features * self.out_features, layers=layers,
                                  seed=seed, latent_init_std=latent_init_std)
        self.weight_scale = float(weight_scale)
        self.gather_output = gather_output
        self.group = group
        self.slice_fn = slice_fn or block_fht_slice
        world, rank = _world(group)
        self.world, self.rank = world, rank
        self.rows = even_shard(self.out_features, rank, world)
        self.row_sizes = [even_shard(self.out_features, r, world)[1] - even_shard(self.out_features, r, world)[0]
                          for r in range(world)]
        self.bias = nn.Parameter(torch.zeros(self.rows[1] - self.rows[0])) if bias else None

    def local_weight(self) -> torch.Tensor:
        r0, r1 = self.rows
        g = self.generator
        latent = _AllReduceGrad.apply(g.latent, self.group)
        w = self.slice_fn(latent, g.size, g.layers, g.seed, r0 * self.in_features, r1 * self.in_features)
        return (w * self.weight_scale).view(r1 - r0, self.in_features)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = F.linear(x, self.local_weight().to(dtype=x.dtype), self.bias)
        if self.gather_output and self.world > 1:
            y = _GatherLastDim.apply(y, self.row_sizes, self.rank, self.group)
        return y


class RowParallelBlockFHTLinear(nn.Module):
    """Input-feature-split BlockFHTLinear: rank r owns W columns [c0, c1).

    Input columns interleave every row of W, so each rank generates the whole
    weight and keeps its columns; the partial products are summed with an
    all-reduce.  ``input_is_parallel`` says x already holds only this rank's
    input features (the output of a ColumnParallel layer).
    """

    def __init__(self, in_features: int, out_features: int, latent_dim: int, layers: int = 3, seed: int = 0,
                 weight_scale: float = 1.0, bias: bool = False, input_is_parallel: bool = True,
                 latent_init_std: float = 0.02, group=None, slice_fn: SliceFn | None = None):
        super().__init__()
        self.in_features, self.out_features = int(in_features), int(out_features)
        self.generator = BlockFHT(int(latent_dim), size=self.in_features * self.out_features, layers=layers,
                                  seed=seed, latent_init_std=latent_init_std)
        self.weight_scale = float(weight_scale)
        self.input_is_parallel = input_is_parallel
        self.group = group
        self.slice_fn = slice_fn or block_fht_slice
        world, rank = _world(group)
        self.world, self.rank = world, rank
        self.cols = even_shard(self.in_features, rank, world)
        self.bias = nn.Parameter(torch.zeros(self.out_features)) if bias else None

    def local_weight(self) -> torch.Tensor:
        c0, c1 = self.cols
        g = self.generator
        latent = _AllReduceGrad.apply(g.latent, self.group)
        w = self.slice_fn(latent, g.size, g.layers, g.seed, 0, g.size) * self.weight_scale
        return w.view(self.out_features, self.in_features)[:, c0:c1]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        c0, c1 = self.cols
        if not self.input_is_parallel:
            x = x[..., c0:c1]
        y = F.linear(x, self.local_weight().to(dtype=x.dtype))
        if self.world > 1:
            y = _AllReduceSum.apply(y, self.group)
        if self.bias is not None:
            y = y + self.bias
        return y


__all__ = ["block_shard", "even_shard", "ShardedBlockFHT", "ColumnParallelBlockFHTLinear",
           "RowParallelBlockFHTLinear", "next_power_of_two"]
