"""Small-block kernel (padded block 2^5 .. 2^10, csrc/fhts.cu) against the CPU oracle.

Every dtype runs fp32 arithmetic here, so the tolerances are tighter than the
tensor-core paths': fp32 1e-5, bf16 / fp16 1e-2 (their output rounding alone
is ~2e-3).  Cases cover whole 1024-coordinate warp tiles, slices that start
and stop inside a tile or inside a 16-byte chunk (the element-wise path),
slices inside one tile, latents shorter than the block, and empty slices.
"""
from __future__ import annotations

import pytest
import torch

from conftest import rel_l2
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 1e-2, torch.float16: 1e-2}
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


@pytest.fixture(scope="module")
def nat(native_lib):
    from latent_weight_lab import _native

    return _native


def _vec(n, seed, dtype, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, generator=g) * scale).to(dtype)


CASES = [
    # (L, size, layers, start, stop)
    (32, 1 << 16, 1, 0, 1 << 16),
    (32, 1 << 16, 3, 0, 1 << 16),
    (17, 5000, 2, 3, 4999),
    (64, 3 * 1024 + 7, 3, 0, 3 * 1024 + 7),
    (100, 40000, 1, 1000, 2000),
    (128, 1 << 15, 2, 8, (1 << 15) - 8),
    (200, 70000, 3, 1029, 1030),
    (256, 1 << 17, 3, 0, 1 << 17),
    (300, 20000, 1, 13, 19991),
    (512, 1 << 16, 1, 4, 1 << 16),
    (777, 1 << 16, 3, 2048, 4096),
    (1024, 1 << 18, 3, 0, 1 << 18),
    (1000, 123457, 2, 511, 123457),
    (1024, 5000, 1, 0, 0),
]


def _ids(c):
    return f"L{c[0]}_s{c[1]}_l{c[2]}_{c[3]}-{c[4]}"


@pytest.mark.parametrize("case", CASES, ids=[_ids(c) for c in CASES])
@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "bf16", "f16"])
def test_small_block_forward(nat, case, dtype):
    L, size, layers, start, stop = case
    z = _vec(L, 11 + L, dtype)
    y = nat.fht_forward(z.cuda(), size, layers, 123, start, stop)
    torch.cuda.synchronize()
    assert y.dtype == dtype and y.shape == (stop - start,)
    if stop == start:
        return
    ref = orc.fht_forward(z.float().numpy(), size, layers, 123, start, stop)
    err = rel_l2(y.float().cpu().numpy(), ref)
    assert err < TOL[dtype], f"forward rel-L2 {err:.3e}"


@pytest.mark.parametrize("case", CASES, ids=[_ids(c) for c in CASES])
@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "bf16", "f16"])
def test_small_block_backward(nat, case, dtype):
    L, size, layers, start, stop = case
    g = _vec(stop - start, 29 + L, dtype)
    grad = nat.fht_backward(g.cuda(), L, size, layers, 123, start, stop)
    torch.cuda.synchronize()
    assert grad.dtype == dtype and grad.shape == (L,)
    ref = orc.fht_backward(g.float().numpy(), L, size, layers, 123, start, stop)
    if stop == start:
        assert float(grad.float().abs().max()) == 0.0
        return
    err = rel_l2(grad.float().cpu().numpy(), ref)
    assert err < TOL[dtype], f"backward rel-L2 {err:.3e}"


@pytest.mark.parametrize("logb", [5, 7, 10])
def test_small_block_unaligned_pointer(nat, logb):
    """A slice view whose data pointer is not 16-byte aligned takes the element-wise path."""
    L = 1 << logb
    size = 1 << 16
    z = _vec(L, 5, torch.bfloat16).cuda()
    full = nat.fht_forward(z, size, 3, 7, 0, size)
    g = _vec(size + 1, 6, torch.bfloat16).cuda()[1:]  # offset by one element
    grad = nat.fht_backward(g, L, size, 3, 7, 0, size)
    torch.cuda.synchronize()
    ref = orc.fht_backward(g.float().cpu().numpy(), L, size, 3, 7, 0, size)
    assert rel_l2(grad.float().cpu().numpy(), ref) < 1e-2
    ref_y = orc.fht_forward(z.float().cpu().numpy(), size, 3, 7, 0, size)
    assert rel_l2(full.float().cpu().numpy(), ref_y) < 1e-2


def test_small_block_deterministic(nat):
    """Two backward calls give bit-identical gradients (fixed summation order)."""
    L, size = 512, 1 << 20
    g = _vec(size, 3, torch.float32).cuda()
    a = nat.fht_backward(g, L, size, 3, 9, 0, size)
    b = nat.fht_backward(g, L, size, 3, 9, 0, size)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_small_block_forced_every_size():
    """Run this file's cases with the kernel forced on for every size and dtype
    it handles (LWL_SMALL_KERNEL=1), including those the default choice gives
    to the tensor-core kernel."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    env = dict(os.environ, LWL_SMALL_KERNEL="1")
    here = Path(__file__).resolve()
    r = subprocess.run([sys.executable, "-m", "pytest", str(here), "-q", "-x", "-k", "not forced", "-p", "no:cacheprovider"],
                       cwd=str(here.parent.parent), env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
