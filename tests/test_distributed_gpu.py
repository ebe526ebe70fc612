"""Block-sharded generation and tensor-parallel BlockFHTLinear on 2 GPUs over NCCL.

Each rank runs the library kernels on its own GPU; results are compared with
a single-GPU computation.  Skipped when fewer than 2 GPUs are visible.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "latent-weight-lab_b200"))
    import torch.distributed as dist

    from latent_weight_lab.block_fht import BlockFHT
    from latent_weight_lab.distributed import ColumnParallelBlockFHTLinear, RowParallelBlockFHTLinear, ShardedBlockFHT

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        z = torch.randn(32768).bfloat16().cuda()
        gen = ShardedBlockFHT(BlockFHT(z.clone(), size=64 * 32768, layers=3, seed=123))
        y = gen()
        lo, hi = gen.shard_range
        torch.manual_seed(1)
        g = torch.randn(64 * 32768).bfloat16().cuda()
        y.backward(g[lo:hi])
        res = {"range": (lo, hi), "y": y.detach().float().cpu(), "grad": gen.generator.latent.grad.float().cpu()}

        torch.manual_seed(3)
        up = ColumnParallelBlockFHTLinear(768, 3072, latent_dim=32768, layers=3, seed=5).cuda()
        down = RowParallelBlockFHTLinear(3072, 768, latent_dim=32768, layers=3, seed=9).cuda()
        torch.manual_seed(4)
        x = torch.randn(64, 768).cuda()
        out = down(torch.nn.functional.gelu(up(x)))
        out.square().sum().backward()
        res.update(out=out.detach().cpu(), gup=up.generator.latent.grad.cpu(), gdown=down.generator.latent.grad.cpu())
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharding_and_tensor_parallel(native_lib):
    from latent_weight_lab import _native
    from latent_weight_lab.block_fht import _BlockFHTLinearFn  # noqa: F401

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0

    # single-GPU reference
    torch.manual_seed(0)
    z = torch.randn(32768).bfloat16().cuda()
    y = _native.fht_forward(z, 64 * 32768, 3, 123, 0, 64 * 32768).float().cpu()
    torch.manual_seed(1)
    g = torch.randn(64 * 32768).bfloat16().cuda()
    grad = _native.fht_backward(g, 32768, 64 * 32768, 3, 123, 0, 64 * 32768).float().cpu()
    got = torch.cat([res[0]["y"], res[1]["y"]])
    assert res[0]["range"] == (0, 32 * 32768)
    assert torch.equal(got, y)
    for r in (0, 1):
        assert (res[r]["grad"] - grad).norm() / grad.norm() < 2e-2  # two bf16 partials summed vs one pass

    from latent_weight_lab import BlockFHTLinear

    torch.manual_seed(3)
    up = BlockFHTLinear(768, 3072, latent_dim=32768, layers=3, seed=5).cuda()
    down = BlockFHTLinear(3072, 768, latent_dim=32768, layers=3, seed=9).cuda()
    torch.manual_seed(4)
    x = torch.randn(64, 768).cuda()
    out = down(torch.nn.functional.gelu(up(x)))
    out.square().sum().backward()
    for r in (0, 1):
        assert (res[r]["out"] - out.detach().cpu()).norm() / out.norm() < 1e-5
        assert (res[r]["gup"] - up.generator.latent.grad.cpu()).norm() / up.generator.latent.grad.norm() < 1e-4
        assert (res[r]["gdown"] - down.generator.latent.grad.cpu()).norm() / down.generator.latent.grad.norm() < 1e-4
