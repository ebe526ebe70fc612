"""The library against the reference's own CUDA extension on the same B200.

oracle/build_ref_ext.py compiles the reference sources (block_fht_ext.cpp,
block_fht_ext_cuda.cu) into oracle/_ref/; that module is the reference's fp32
GPU transform (csrc/block_fht_ext_cuda.cu:516-622) and fused linear
(:624-681).  Here it is a second checker beside the CPU oracle: fp32 outputs
and latent gradients agree within 1e-5 relative L2 (the reference builds with
--use_fast_math and sums the backward with atomics), and the fused linear
agrees where the reference's fused kernel applies.  The timing test prints one
JSON line per point (run with -s) and asserts nothing about speed.
Skipped when oracle/_ref has not been built.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import json
from pathlib import Path

import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu

SO = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "lwl_ref_block_fht_ext.so"


@pytest.fixture(scope="module")
def ref():
    if not SO.exists():
        pytest.skip("oracle/_ref not built (python oracle/build_ref_ext.py)")
    loader = importlib.machinery.ExtensionFileLoader("lwl_ref_block_fht_ext", str(SO))
    spec = importlib.util.spec_from_loader("lwl_ref_block_fht_ext", loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def nat(native_lib):
    from latent_weight_lab import _native

    return _native


def _one(r):
    return r[0] if isinstance(r, (list, tuple)) else r


CASES = [
    # (L, size, layers, seed, start, stop): the reference's shared-memory path
    # (B <= 16384) and its global multi-pass path (larger B)
    (1024, 108618, 3, 123, 0, 108618),
    (1024, 108618, 3, 123, 1000, 2000),
    (100, 70000, 1, 5, 3, 69999),
    (5000, 40000, 2, 7, 17, 39990),
    (16384, 5 * 16384, 3, 9, 0, 5 * 16384),
    (32768, 3 * 32768, 3, 11, 5, 3 * 32768 - 5),
    (200000, 600000, 2, 13, 1234, 598765),
]


@pytest.mark.parametrize("case", CASES, ids=[f"L{c[0]}_s{c[1]}_l{c[2]}" for c in CASES])
def test_matches_reference_cuda(ref, nat, case):
    L, size, layers, seed, start, stop = case
    z = torch.randn(L, generator=torch.Generator().manual_seed(L)).cuda()
    y_ref = _one(ref.forward(z, size, layers, seed, start, stop))
    y = nat.fht_forward(z, size, layers, seed, start, stop)
    g = torch.randn(stop - start, generator=torch.Generator().manual_seed(L + 1)).cuda()
    gz_ref = _one(ref.backward(g, L, size, layers, seed, start, stop))
    gz = nat.fht_backward(g, L, size, layers, seed, start, stop)
    torch.cuda.synchronize()
    assert rel_l2(y.cpu().numpy(), y_ref.cpu().numpy()) < 1e-5
    assert rel_l2(gz.cpu().numpy(), gz_ref.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_linear_matches_reference_cuda(ref, dtype):
    """Where the reference's fused kernel runs (B <= 16384, B % in == 0)."""
    from latent_weight_lab import block_fht_linear_forward

    torch.manual_seed(3)
    T, K, N, L = 256, 512, 384, 8192
    x = torch.randn(T, K, device="cuda").to(dtype)
    z = (torch.randn(L, device="cuda") * 0.02).to(dtype)
    y_ref = _one(ref.linear_forward(x, z, N, 3, 21, 1.0))
    y = block_fht_linear_forward(x, z, N, 3, 21)
    torch.cuda.synchronize()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert rel_l2(y.float().cpu().numpy(), y_ref.float().cpu().numpy()) < tol


def _time(fn, reps=3):
    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


@pytest.mark.parametrize("logb", [10, 14, 15, 18])
@pytest.mark.parametrize("layers", [1, 3])
def test_time_against_reference_cuda(ref, nat, logb, layers):
    """fp32, 2^26 coordinates per call, latent length = block size (the C2 sweep's shape)."""
    B, N = 1 << logb, 1 << 26
    z = torch.randn(B, device="cuda")
    g = torch.randn(N, device="cuda")
    res = {"dtype": "fp32", "block_size": B, "layers": layers, "coords": N}
    for name, fwd, bwd in (
        ("reference_cuda", lambda: ref.forward(z, N, layers, 123, 0, N), lambda: ref.backward(g, B, N, layers, 123, 0, N)),
        ("ours", lambda: nat.fht_forward(z, N, layers, 123, 0, N), lambda: nat.fht_backward(g, B, N, layers, 123, 0, N)),
    ):
        res[name] = {"forward_gcoords_s": N / _time(fwd) / 1e6, "backward_gcoords_s": N / _time(bwd) / 1e6}
    print(json.dumps(res), flush=True)
