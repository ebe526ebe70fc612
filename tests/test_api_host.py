"""Host-side behaviour of the drop-in Python API that needs no GPU."""
from __future__ import annotations

import pytest
import torch

import latent_weight_lab as lwl
from latent_weight_lab import block_fht as bf


def test_public_names_match_reference_package():
    expected = {"BlockFHT", "BlockFHTLinear", "block_fht_linear_forward", "block_fht_slice",
                "flush_block_fht_weight_cache", "prepare_block_fht_weight_cache",
                "restore_block_fht_weight_cache", "sign_word_for", "suspend_block_fht_weight_cache"}
    assert expected <= set(lwl.__all__)


def test_scalar_sign_word_matches_golden(golden):
    for point, word in zip(golden["sign_points"], golden["sign_words"]):
        assert bf.sign_word_for(*[int(v) for v in point]) == int(word)


def test_sign_word_uses_32_positions():
    bits = bf.sign_word_for(seed=999, block=3, layer=2, word=4)
    signs = [1 if ((bits >> b) & 1) else -1 for b in range(32)]
    assert len(signs) == 32 and set(signs) <= {-1, 1}


def test_block_size_metadata():
    assert bf.BlockFHT(32, size=64, layers=1, seed=1).block_size == 32
    assert bf.BlockFHT((1 << 23) - 17, size=1 << 23, layers=1, seed=1).block_size == 1 << 23
    assert bf.BlockFHT(7, size=31, layers=2).block_size == 8


def test_constructor_validation_messages():
    with pytest.raises(ValueError, match="size must be positive"):
        bf.BlockFHT(8, size=0)
    with pytest.raises(ValueError, match="layers must be 1, 2, or 3"):
        bf.BlockFHT(8, size=10, layers=4)
    with pytest.raises(ValueError, match="latent size must be positive"):
        bf.BlockFHT(0, size=10)
    with pytest.raises(ValueError, match="latent tensor must be 1D"):
        bf.BlockFHT(torch.zeros(2, 2), size=10)
    with pytest.raises(ValueError, match="value must be positive"):
        bf.next_power_of_two(0)
    with pytest.raises(ValueError, match="spectral_rank exceeds"):
        bf.BlockFHTLinear(4, 4, latent_dim=8, spectral_rank=5)


def test_external_latent_parameter_identity():
    latent = torch.nn.Parameter(torch.randn(8))
    assert bf.BlockFHT(latent, size=40, layers=1, seed=5).latent is latent


def test_state_dict_keys_match_reference_layout():
    layer = bf.BlockFHTLinear(5, 3, bias=True, latent_dim=8, layers=2, seed=11, output_gain=True, input_gain=True)
    assert set(layer.state_dict()) == {"generator.latent", "bias", "output_gain", "input_gain"}
    spec = bf.BlockFHTLinear(8, 12, latent_dim=8, spectral_rank=2, spectral_out_groups=3, spectral_in_groups=2)
    assert {"spectral_u", "spectral_v", "spectral_core"} <= set(spec.state_dict())


def test_default_latent_dim_from_ratio():
    layer = bf.BlockFHTLinear(768, 3072)
    assert layer.generator.latent_size == round(768 * 3072 * 0.01)
    assert layer.generator.block_size == 32768


def test_cpu_tensors_raise_instead_of_falling_back():
    g = bf.BlockFHT(8, size=40, layers=1, seed=5)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        g()


def test_invalid_slice_message():
    g = bf.BlockFHT(8, size=40, layers=1, seed=5)
    with pytest.raises(ValueError, match=r"invalid slice \[5, 41\) for size 40"):
        g.slice(5, 41)
