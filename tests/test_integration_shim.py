"""The ctypes shim shown in INTEGRATION.md (reference-side binding) works against the library."""
from __future__ import annotations

from pathlib import Path

import pytest
import torch

from conftest import rel_l2
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _shim_class():
    """Execute the ctypes shim exactly as INTEGRATION.md prints it."""
    text = (Path(__file__).resolve().parents[1] / "INTEGRATION.md").read_text()
    sec = text[text.index("## Reference-side binding"):]
    code = sec[sec.index("```python") + len("```python"):]
    code = code[:code.index("```")]
    ns: dict = {}
    exec(compile(code, "INTEGRATION.md", "exec"), ns)
    return ns["_LwlB200Ext"]


def test_shim_matches_oracle(native_lib):
    from latent_weight_lab import _native

    ext = _shim_class()(str(_native.library_path()))
    torch.manual_seed(0)
    z = torch.randn(1024, device="cuda")
    y = ext.forward(z, 108618, 3, 123, 0, 108618)[0]
    assert rel_l2(y.cpu().numpy(), orc.fht_forward(z.cpu().numpy(), 108618, 3, 123, 0, 108618)) < 1e-5
    g = torch.randn(108618, device="cuda")
    grad = ext.backward(g, 1024, 108618, 3, 123, 0, 108618)
    ref = orc.fht_backward(g.cpu().numpy(), 1024, 108618, 3, 123, 0, 108618)
    assert rel_l2(grad.cpu().numpy(), ref) < 1e-5
    x = torch.randn(5, 8, device="cuda")
    out = ext.linear_forward(x, torch.randn(32, device="cuda"), 6, 2, 9, 0.5)
    assert out.shape == (5, 6)


def test_shim_fused_linear_bf16(native_lib):
    """bf16 768 -> 3072 goes through lwl_linear_forward and matches the oracle."""
    from latent_weight_lab import _native

    ext = _shim_class()(str(_native.library_path()))
    torch.manual_seed(1)
    x = torch.randn(200, 768, device="cuda").bfloat16()
    z = (torch.randn(32768) * 0.02).bfloat16()
    y = ext.linear_forward(x, z.cuda(), 3072, 3, 4, 0.5)
    direct = _native.linear_forward(x, z.cuda(), 3072, 3, 4, 0.5)
    assert torch.equal(y, direct)
    ref = orc.linear_forward(x.float().cpu().numpy(), z.float().numpy(), 3072, 3, 4, 0.5)
    assert rel_l2(y.float().cpu().numpy(), ref) < 1e-2
