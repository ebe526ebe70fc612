"""bf16 forward plans of large blocks (2^18 .. 2^23) keep their workspace in
bf16 and stream it into the low pass by bulk copy (csrc/fht_engine.cu,
fht_lo_kernel).  Checked here through the C ABI: the workspace size query,
the 16-byte alignment the bulk copy needs, and agreement with the fp32
workspace plan (LWL_WS16=0) and the oracle."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from conftest import rel_l2
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

LWL_BF16 = 1


@pytest.fixture(scope="module")
def lib(native_lib):
    return native_lib


def _call(lib, z, size, layers, seed, start, stop, ws, ws_bytes):
    out = torch.empty(stop - start, device="cuda", dtype=torch.bfloat16)
    st = lib.lwl_fht_forward(LWL_BF16, z.data_ptr(), z.numel(), size, layers, seed, start, stop, out.data_ptr(),
                             ws, ws_bytes, 0, torch.cuda.current_stream().cuda_stream)
    return st, out


@pytest.mark.parametrize("logb, layers", [(18, 1), (18, 3), (20, 2), (22, 3)])
def test_bf16_workspace_forward(lib, logb, layers):
    B = 1 << logb
    size, start, stop = 3 * B, 1000, 3 * B - 7
    z = (torch.randn(B, generator=torch.Generator().manual_seed(logb)) * 3).bfloat16()
    zc = z.cuda()
    need = lib.lwl_fht_forward_workspace_bytes(LWL_BF16, B, size, layers, start, stop, 0)
    assert need == 3 * B * 2  # two bytes per coordinate of the touched blocks
    ws = torch.empty(need + 16, dtype=torch.uint8, device="cuda")
    st, out = _call(lib, zc, size, layers, 5, start, stop, ws.data_ptr(), need)
    torch.cuda.synchronize()
    assert st == 0, lib.lwl_last_error()
    ref = orc.fht_forward(z.float().numpy(), size, layers, 5, start, stop)
    assert rel_l2(out.float().cpu().numpy(), ref) < 1e-2
    # a workspace that is not 16-byte aligned is refused before anything runs
    st, _ = _call(lib, zc, size, layers, 5, start, stop, ws.data_ptr() + 2, need)
    assert st == 1 and b"16-byte aligned" in lib.lwl_last_error()


def test_bf16_workspace_matches_fp32_workspace():
    """The same call with the fp32 workspace plan (LWL_WS16=0, another process)."""
    code = r"""
import sys, torch
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/latent-weight-lab_b200"]
from latent_weight_lab import _native
z = (torch.randn(1 << 19, generator=torch.Generator().manual_seed(3))).bfloat16().cuda()
y = _native.fht_forward(z, 2 << 19, 3, 9, 0, 2 << 19)
torch.save(y.float().cpu(), sys.argv[2])
"""
    repo = Path(__file__).resolve().parent.parent
    outs = []
    for flag in ("1", "0"):
        path = repo / "gpurun_out" / f"_ws16_{flag}.pt"
        path.parent.mkdir(exist_ok=True)
        env = dict(os.environ, LWL_WS16=flag)
        r = subprocess.run([sys.executable, "-c", code, str(repo), str(path)], env=env, capture_output=True,
                           text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.append(torch.load(path))
        path.unlink()
    a, b = outs
    # one extra bf16 rounding per launch: well inside the bf16 gate
    assert float((a - b).norm() / b.norm()) < 5e-3
