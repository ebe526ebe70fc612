"""FixedFHTMix: oracle and signs pinned to the reference's outputs (CPU), the
CUDA kernel against them (GPU)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden_fht_mix.npz"


def _cases():
    g = np.load(GOLDEN)
    for i in range(int(g["count"])):
        features, seed, rows = (int(v) for v in g[f"mix{i}_meta"])
        yield features, seed, rows, g[f"mix{i}_signs"], g[f"mix{i}_x"], g[f"mix{i}_g"], g[f"mix{i}_y"], g[f"mix{i}_gx"]


def test_oracle_matches_reference_fixtures():
    for features, _, _, signs, x, gy, y, gx in _cases():
        assert rel_l2(orc.fixed_fht_mix(x, signs), y) < 1e-6, features
        # the map is its own adjoint: the input gradient is the same map on g
        assert rel_l2(orc.fixed_fht_mix(gy, signs), gx) < 1e-6, features


def test_module_signs_match_reference():
    from latent_weight_lab.fht_mix import FixedFHTMix

    for features, seed, _, signs, *_ in _cases():
        mix = FixedFHTMix(features, seed)
        assert mix.padded == signs.size
        assert np.array_equal(mix.signs.numpy(), signs)
        assert "signs" in mix.state_dict()


def test_module_rejects_wrong_width():
    from latent_weight_lab.fht_mix import FixedFHTMix

    with pytest.raises(ValueError, match="expected last dim 24, got 25"):
        FixedFHTMix(24, 1)(torch.zeros(2, 25))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype, tol", [(torch.float32, 1e-5), (torch.bfloat16, 1e-2), (torch.float16, 1e-2)])
def test_gpu_forward_backward_match_reference(native_lib, dtype, tol):
    from latent_weight_lab.fht_mix import FixedFHTMix

    for features, seed, rows, signs, x, gy, y, gx in _cases():
        mix = FixedFHTMix(features, seed).cuda()
        xt = torch.from_numpy(x).cuda().to(dtype).requires_grad_(True)
        out = mix(xt)
        out.backward(torch.from_numpy(gy).cuda().to(dtype))
        if dtype == torch.float32:
            ref_y, ref_gx = y, gx
        else:  # fp32 math on the rounded inputs, rounded once
            ref_y = orc.fixed_fht_mix(xt.detach().float().cpu().numpy(), signs)
            ref_gx = orc.fixed_fht_mix(torch.from_numpy(gy).to(dtype).float().numpy(), signs)
        assert out.dtype == dtype and out.shape == (rows, features)
        assert rel_l2(out.detach().float().cpu().numpy(), ref_y) < tol, features
        assert rel_l2(xt.grad.float().cpu().numpy(), ref_gx) < tol, features


@pytest.mark.gpu
@pytest.mark.parametrize("features", [1, 5, 8, 16, 24, 31, 32, 33, 40, 64, 100, 128, 200, 520, 768, 1024, 1025, 1600,
                                      2048, 2049, 3072, 4095, 6400, 8191, 8192])
def test_gpu_shapes_against_oracle(native_lib, features):
    """Every register/shuffle/exchange regime, ragged widths, leading dims, many rows."""
    from latent_weight_lab.fht_mix import FixedFHTMix

    torch.manual_seed(features)
    mix = FixedFHTMix(features, features + 3).cuda()
    x = torch.randn(3, 37, features, device="cuda")
    y = mix(x)
    ref = orc.fixed_fht_mix(x.cpu().numpy(), mix.signs.cpu().numpy())
    assert rel_l2(y.cpu().numpy(), ref) < 1e-5
    assert torch.allclose(mix(mix(x)), x, atol=1e-4) or features & (features - 1)  # involution when P == F


@pytest.mark.gpu
@pytest.mark.parametrize("features", [8, 16, 24, 56, 136, 768, 1000, 1600, 3072, 6400])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gpu_wide_rows_half(native_lib, features, dtype):
    """16-bit rows at the GPT widths and at other 16-byte-aligned widths (the prefetching tile
    kernel for P >= 128): 1e-2 against fp32 math on the rounded input."""
    from latent_weight_lab.fht_mix import FixedFHTMix

    torch.manual_seed(features + 1)
    mix = FixedFHTMix(features, 11).cuda()
    x = torch.randn(257, features, device="cuda").to(dtype)
    y = mix(x)
    ref = orc.fixed_fht_mix(x.float().cpu().numpy(), mix.signs.cpu().numpy())
    assert y.dtype == dtype
    assert rel_l2(y.float().cpu().numpy(), ref) < 1e-2


@pytest.mark.gpu
def test_gpu_normalized_fht_and_wrappers(native_lib):
    from latent_weight_lab.fht_mix import (FixedFHTInputMixLinear, FixedFHTOutputMixLinear, normalized_fht_last_dim)

    torch.manual_seed(0)
    v = torch.randn(5, 256, device="cuda")
    assert rel_l2(normalized_fht_last_dim(v).cpu().numpy(), orc.normalized_wht_last_dim(v.cpu().numpy())) < 1e-6
    with pytest.raises(ValueError):
        normalized_fht_last_dim(torch.zeros(2, 12, device="cuda"))
    lin = torch.nn.Linear(64, 96).cuda()
    x = torch.randn(7, 64, device="cuda")
    outm = FixedFHTOutputMixLinear(lin, 96, 4).cuda()
    ref = orc.fixed_fht_mix(lin(x).detach().cpu().numpy(), outm.mix.signs.cpu().numpy())
    assert rel_l2(outm(x).detach().cpu().numpy(), ref) < 1e-5
    inm = FixedFHTInputMixLinear(lin, 64, 9).cuda()
    mixed = torch.from_numpy(orc.fixed_fht_mix(x.cpu().numpy(), inm.mix.signs.cpu().numpy()).astype(np.float32)).cuda()
    assert rel_l2(inm(x).detach().cpu().numpy(), lin(mixed).detach().cpu().numpy()) < 1e-5
