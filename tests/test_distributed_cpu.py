"""Multi-rank logic of latent_weight_lab.distributed on 2 gloo ranks (CPU).

The sharding, the collectives and the gradient wiring are product code; the
per-rank generator evaluation is replaced by the CPU oracle (test
infrastructure) through the modules' slice_fn hook, since the library kernels
need a GPU.  Results are compared with a single-process oracle computation.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as orc


class _OracleSlice(torch.autograd.Function):
    @staticmethod
    def forward(ctx, latent, size, layers, seed, start, stop):
        ctx.args = (latent.numel(), size, layers, seed, start, stop)
        return torch.from_numpy(orc.fht_forward(latent.detach().numpy(), size, layers, seed, start, stop))

    @staticmethod
    def backward(ctx, g):
        L, size, layers, seed, start, stop = ctx.args
        grad = orc.fht_backward(g.contiguous().numpy(), L, size, layers, seed, start, stop)
        return torch.from_numpy(grad), None, None, None, None, None


def oracle_slice(latent, size, layers, seed, start, stop):
    return _OracleSlice.apply(latent, size, layers, seed, start, stop)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fn, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, fn(rank, world)))
    finally:
        dist.destroy_process_group()


def run_ranks(fn, world=2):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return [out[r] for r in range(world)]


def test_block_shard_covers_every_coordinate_once():
    from latent_weight_lab.distributed import block_shard

    for size, B, world in [(108618, 1024, 2), (2**28, 32768, 8), (100, 32, 3), (5, 8, 4)]:
        ranges = [block_shard(size, B, r, world) for r in range(world)]
        assert ranges[0][0] == 0 and ranges[-1][1] == size
        for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
            assert a1 == b0
        for lo, hi in ranges:
            assert lo % B == 0 and lo <= hi


def _sharded_generator(rank, world):
    from latent_weight_lab.block_fht import BlockFHT
    from latent_weight_lab.distributed import ShardedBlockFHT

    torch.manual_seed(0)
    z = torch.randn(1024)
    gen = ShardedBlockFHT(BlockFHT(z.clone(), size=108618, layers=3, seed=123), slice_fn=oracle_slice)
    y = gen()
    torch.manual_seed(1)
    g = torch.randn(108618)
    lo, hi = gen.shard_range
    (y * g[lo:hi]).sum().backward()
    return gen.shard_range, y.detach().numpy(), gen.generator.latent.grad.numpy()


def test_sharded_generator_matches_single_process():
    res = run_ranks(_sharded_generator)
    torch.manual_seed(0)
    z = torch.randn(1024).numpy()
    torch.manual_seed(1)
    g = torch.randn(108618).numpy()
    full = orc.fht_forward(z, 108618, 3, 123, 0, 108618)
    grad = orc.fht_backward(g, 1024, 108618, 3, 123, 0, 108618)
    got = np.concatenate([r[1] for r in res])
    assert res[0][0][0] == 0 and res[-1][0][1] == 108618
    assert np.array_equal(got, full)
    for r in res:  # every rank holds the all-reduced latent gradient
        assert np.allclose(r[2], grad, rtol=1e-5, atol=1e-5)


def _tp_mlp(rank, world):
    from latent_weight_lab.distributed import ColumnParallelBlockFHTLinear, RowParallelBlockFHTLinear

    torch.manual_seed(3)
    up = ColumnParallelBlockFHTLinear(24, 40, latent_dim=100, layers=2, seed=5, slice_fn=oracle_slice)
    down = RowParallelBlockFHTLinear(40, 24, latent_dim=60, layers=3, seed=9, slice_fn=oracle_slice)
    torch.manual_seed(4)
    x = torch.randn(6, 24)
    y = down(F_gelu(up(x)))
    y.square().sum().backward()
    return y.detach().numpy(), up.generator.latent.grad.numpy(), down.generator.latent.grad.numpy()


def F_gelu(t):
    return torch.nn.functional.gelu(t)


def test_tensor_parallel_mlp_matches_single_process():
    res = run_ranks(_tp_mlp)
    # single-process reference with the same initial latents
    torch.manual_seed(3)
    z_up = torch.randn(100) * 0.02
    z_down = torch.randn(60) * 0.02
    up_l = z_up.clone().requires_grad_(True)
    down_l = z_down.clone().requires_grad_(True)
    torch.manual_seed(4)
    x = torch.randn(6, 24)
    w_up = oracle_slice(up_l, 24 * 40, 2, 5, 0, 960).view(40, 24)
    w_down = oracle_slice(down_l, 40 * 24, 3, 9, 0, 960).view(24, 40)
    y = torch.nn.functional.gelu(x @ w_up.T) @ w_down.T
    y.square().sum().backward()
    for yr, gu, gd in res:
        assert np.allclose(yr, y.detach().numpy(), rtol=1e-5, atol=1e-6)
        assert np.allclose(gu, up_l.grad.numpy(), rtol=1e-4, atol=1e-6)
        assert np.allclose(gd, down_l.grad.numpy(), rtol=1e-4, atol=1e-6)
