"""lwl_fht_backward_noalloc: the latent-gradient entry point for callers that cannot allocate.

Some callers have no device allocator at hand (for example a plugin driven by
a host runtime that owns all device memory), so this entry point keeps its
scratch partials in a fixed array inside the library instead of taking a
workspace.  The test checks, through the C ABI, that it returns the same
gradient as lwl_fht_backward on two calls in a row (the array keeps the
previous call's contents, so the second call must not depend on them), and
checks it against the CPU oracle directly, for fp32, bf16 and fp16 and for a
call with more blocks than the array has partial rows (the CTA cap).
Collected last so a stop-at-first-failure run has already run every other test.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import rel_l2
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _noalloc(lib):
    fn = lib.lwl_fht_backward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_uint64,
                   ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_uint, ctypes.c_void_p]
    return fn


@pytest.mark.parametrize("L, size, layers, start, stop", [
    (4096, 20000, 3, 0, 20000),
    (16384, 40 * 16384, 2, 777, 39 * 16384 + 5),
    (100, 5000, 1, 17, 4999),
])
def test_noalloc_backward_matches_workspace_backward(native_lib, L, size, layers, start, stop):
    from latent_weight_lab import _native

    fn = _noalloc(native_lib)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        g = torch.randn(stop - start, device="cuda", generator=torch.Generator("cuda").manual_seed(call))
        ref = _native.fht_backward(g, L, size, layers, 123 + call, start, stop)
        got = torch.full((L,), float("nan"), device="cuda")
        st = fn(_native.LWL_F32, g.data_ptr(), L, size, layers, 123 + call, start, stop, got.data_ptr(), 0, stream)
        assert st == 0, native_lib.lwl_last_error()
        torch.cuda.synchronize()
        assert rel_l2(got.cpu().numpy(), ref.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16], ids=["f32", "bf16", "f16"])
@pytest.mark.parametrize("L, size, layers, start, stop", [
    (16384, 320 * 16384, 3, 5, 320 * 16384 - 9),  # 320 blocks > the 128 partial rows the array holds at L = 16384
    (3000, 50000, 2, 0, 50000),
])
def test_noalloc_backward_against_oracle(native_lib, dtype, L, size, layers, start, stop):
    """Absolute parity with the oracle (fp32 1e-5, 16-bit 1e-2 against fp32 math on the rounded input)."""
    from latent_weight_lab import _native

    fn = _noalloc(native_lib)
    code = {torch.float32: _native.LWL_F32, torch.bfloat16: _native.LWL_BF16, torch.float16: _native.LWL_F16}[dtype]
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        g = torch.randn(stop - start, generator=torch.Generator().manual_seed(10 + call)).to(dtype)
        ref = orc.fht_backward(g.float().numpy(), L, size, layers, 321 + call, start, stop)
        gd = g.cuda()
        got = torch.full((L,), float("nan"), device="cuda", dtype=dtype)
        st = fn(code, gd.data_ptr(), L, size, layers, 321 + call, start, stop, got.data_ptr(), 0, stream)
        assert st == 0, native_lib.lwl_last_error()
        assert native_lib.lwl_last_error() == b""
        torch.cuda.synchronize()
        assert rel_l2(got.float().cpu().numpy(), ref) < tol


def test_noalloc_rejects_large_blocks(native_lib):
    fn = _noalloc(native_lib)
    g = torch.zeros(10, device="cuda")
    out = torch.zeros(32768, device="cuda")
    st = fn(0, g.data_ptr(), 32768, 65536, 3, 1, 0, 10, out.data_ptr(), 0, None)
    assert st == 2
    assert b"2^14" in native_lib.lwl_last_error()
