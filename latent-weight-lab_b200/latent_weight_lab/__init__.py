"""latent_weight_lab -- B200-native BlockFHT generator (drop-in for the reference package)."""
from .block_fht import (
    BlockFHT,
    BlockFHTLinear,
    block_fht_grad_latent,
    block_fht_linear_forward,
    block_fht_slice,
    exact_arithmetic,
    flush_block_fht_weight_cache,
    next_power_of_two,
    prepare_block_fht_weight_cache,
    restore_block_fht_weight_cache,
    sign_word_for,
    signs_for,
    suspend_block_fht_weight_cache,
)

__all__ = [
    "BlockFHT",
    "BlockFHTLinear",
    "block_fht_linear_forward",
    "block_fht_slice",
    "flush_block_fht_weight_cache",
    "prepare_block_fht_weight_cache",
    "restore_block_fht_weight_cache",
    "sign_word_for",
    "suspend_block_fht_weight_cache",
]
