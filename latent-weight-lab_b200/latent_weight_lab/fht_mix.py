"""Fixed sign-Hadamard activation mixing on liblwl_b200.

``FixedFHTMix`` (reference ``examples/nanogpt/model.py:200-218``) maps the last
dimension of its input through ``S * H_P / sqrt(P) * S`` on the zero-padded
vector and keeps the first ``features`` entries, P = next_pow2(features), with
a fixed +-1 sign vector ``S`` drawn from ``torch.Generator().manual_seed(seed)``
exactly as the reference does (same buffer name ``signs``, persistent).  The
map is its own adjoint, so the backward is the same kernel applied to the
upstream gradient.  ``FixedFHTOutputMixLinear`` / ``FixedFHTInputMixLinear``
(``model.py:221-238``) wrap a linear with it.  CUDA tensors only.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _native
from .block_fht import next_power_of_two

__all__ = ["FixedFHTMix", "FixedFHTOutputMixLinear", "FixedFHTInputMixLinear", "normalized_fht_last_dim"]


class _FixedFHTMixFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, signs):
        ctx.save_for_backward(signs)
        return _native.fixed_fht_mix(x, signs)

    @staticmethod
    def backward(ctx, grad_y):
        (signs,) = ctx.saved_tensors
        return _native.fixed_fht_mix(grad_y, signs), None


def normalized_fht_last_dim(values: torch.Tensor) -> torch.Tensor:
    """Natural-order Walsh-Hadamard over the last dimension times 1/sqrt(n)
    (model.py:182-197); n must be a power of two (<= 8192 here)."""
    size = values.shape[-1]
    if size & (size - 1):
        raise ValueError("FHT size must be a power of two")
    ones = torch.ones(size, device=values.device, dtype=torch.float32)
    return _FixedFHTMixFn.apply(values, ones)


class FixedFHTMix(nn.Module):
    def __init__(self, features: int, seed: int) -> None:
        super().__init__()
        self.features = int(features)
        self.padded = next_power_of_two(self.features)
        generator = torch.Generator(device="cpu")
        generator.manual_seed(int(seed))
        signs = torch.randint(0, 2, (self.padded,), generator=generator, dtype=torch.float32) * 2.0 - 1.0
        self.register_buffer("signs", signs, persistent=True)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.features:
            raise ValueError(f"expected last dim {self.features}, got {x.shape[-1]}")
        return _FixedFHTMixFn.apply(x, self.signs)


class FixedFHTOutputMixLinear(nn.Module):
    def __init__(self, linear: nn.Module, out_features: int, seed: int) -> None:
        super().__init__()
        self.linear = linear
        self.mix = FixedFHTMix(out_features, seed)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.mix(self.linear(x))


class FixedFHTInputMixLinear(nn.Module):
    def __init__(self, linear: nn.Module, in_features: int, seed: int) -> None:
        super().__init__()
        self.mix = FixedFHTMix(in_features, seed)
        self.linear = linear

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.linear(self.mix(x))
