"""tcgen05 BlockFHTLinear forward: the dense-weight pipeline and the fused generator path.

Tolerance: rel-L2 1e-2 against fp32 math (bf16 operands, fp32 accumulation,
bf16 output; the fused weight is also compared with the fp32 oracle weight
on the same bf16 latent).
"""
from __future__ import annotations

import pytest
import torch

from conftest import rel_l2
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T, K, N", [(256, 768, 256), (1000, 64, 128), (130, 512, 384), (3000, 768, 1024)])
def test_dense_pipeline_matches_matmul(native_lib, T, K, N):
    from latent_weight_lab import _native

    torch.manual_seed(T + K + N)
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda").bfloat16()
    y, err = _native.tc_linear_dense(x, w)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = x.float() @ w.float().T
    assert rel_l2(y.float().cpu().numpy(), ref.cpu().numpy()) < 1e-2


@pytest.mark.parametrize("K, N, L, layers", [(768, 3072, 32768, 3), (768, 768, 5898, 3), (512, 256, 1000, 1),
                                             (256, 384, 20000, 2), (768, 2304, 17694, 3)])
def test_fused_forward_matches_oracle_weight(native_lib, K, N, L, layers):
    from latent_weight_lab import _native

    torch.manual_seed(K + N + L)
    T = 777
    x = torch.randn(T, K, device="cuda").bfloat16()
    z = (torch.randn(L) * 0.02).bfloat16()
    out = _native.linear_forward(x, z.cuda(), N, layers, 5 + layers, weight_scale=0.5, return_status=True)
    assert out is not None
    y, err = out
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    w = torch.from_numpy(orc.generated_weight(z.float().numpy(), K, N, layers, 5 + layers, 0.5)).cuda()
    ref = x.float() @ w.T
    assert rel_l2(y.float().cpu().numpy(), ref.cpu().numpy()) < 1e-2


def test_fused_forward_unsupported_shape_returns_none(native_lib):
    from latent_weight_lab import _native

    x = torch.randn(16, 100, device="cuda").bfloat16()
    assert _native.linear_forward(x, torch.randn(300, device="cuda").bfloat16(), 128, 3, 1) is None
