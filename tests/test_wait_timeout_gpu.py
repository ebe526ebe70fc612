"""Failure detection on the GPU without a fault: a bounded device wait that runs out.

The tensor-core backward fetches each gradient block with a bulk copy and
waits on an mbarrier with a bounded number of polls.  LWL_FLAG_TEST_WAIT_TIMEOUT
leaves the first copy of every CTA unissued (so nothing is in flight) and
shortens the bound, so every wait gives up.  The kernel records the failure
in the workspace's error word and poisons the result with NaN; the host reads
the status with lwl_fht_backward_status, and the context stays usable: the
next ordinary call on the same workspace succeeds and matches the oracle.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import rel_l2
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def test_backward_wait_timeout_is_reported(native_lib):
    from latent_weight_lab import _native

    lib = native_lib
    B, nblk, layers, seed = 32768, 8, 3, 17
    size = B * nblk
    code = _native.LWL_BF16
    g = torch.randn(size, generator=torch.Generator().manual_seed(1)).bfloat16()
    gd = g.cuda()
    ws_bytes = lib.lwl_fht_backward_workspace_bytes(code, B, size, layers, 0, size, 0)
    assert ws_bytes > 0
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty(B, dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    st = lib.lwl_fht_backward(code, gd.data_ptr(), B, size, layers, seed, 0, size, out.data_ptr(), ws.data_ptr(),
                              ws_bytes, _native.FLAG_TEST_WAIT_TIMEOUT, stream)
    assert st == 0, lib.lwl_last_error()  # the launch itself succeeds; the failure is on the device
    status = lib.lwl_fht_backward_status(code, B, size, layers, 0, size, 0, ws.data_ptr(), stream)
    assert status == 5, (status, lib.lwl_last_error())  # LWL_ERR_TIMEOUT
    assert b"gave up" in lib.lwl_last_error()
    assert torch.isnan(out.float()).all()

    # the context is still usable: an ordinary call on the same workspace works
    st = lib.lwl_fht_backward(code, gd.data_ptr(), B, size, layers, seed, 0, size, out.data_ptr(), ws.data_ptr(),
                              ws_bytes, 0, stream)
    assert st == 0, lib.lwl_last_error()
    assert lib.lwl_fht_backward_status(code, B, size, layers, 0, size, 0, ws.data_ptr(), stream) == 0
    ref = orc.fht_backward(g.float().numpy(), B, size, layers, seed, 0, size)
    assert rel_l2(out.float().cpu().numpy(), ref) < 1e-2


def test_linear_forward_status_ok(native_lib):
    from latent_weight_lab import _native

    lib = native_lib
    x = torch.randn(256, 768, device="cuda").bfloat16()
    z = (0.02 * torch.randn(32768, device="cuda")).bfloat16()
    ws = torch.zeros(lib.lwl_linear_forward_workspace_bytes(), dtype=torch.uint8, device="cuda")
    y = torch.empty(256, 3072, device="cuda", dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    st = lib.lwl_linear_forward(_native.LWL_BF16, x.data_ptr(), 256, 768, z.data_ptr(), 32768, 3072, 3, 5,
                                ctypes.c_float(1.0), y.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    assert st == 0, lib.lwl_last_error()
    assert lib.lwl_linear_forward_status(ws.data_ptr(), stream) == 0
