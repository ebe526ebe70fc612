"""The CPU oracle against golden vectors recorded from the reference implementation."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2
from oracle import oracle as orc

# Known answers computed from the reference (sign_word_for, block_fht.py:46-52).
KNOWN_WORDS = {
    (0, 0, 0, 0): 0x80059753,
    (123, 0, 0, 0): 0x87D01FB1,
    (123, 106, 3, 31): 0xB4258089,
    (999, 3, 2, 4): 0x2140A4D8,
    (2**40 + 5, 8191, 2, 1023): 0xD150C333,
    (-1, 1, 1, 1): 0x05C18E34,
}


def test_known_sign_words():
    for args, word in KNOWN_WORDS.items():
        assert orc.sign_word(*args) == word


def test_sign_words_match_golden_table(golden):
    for point, word in zip(golden["sign_points"], golden["sign_words"]):
        assert orc.sign_word(*[int(v) for v in point]) == int(word)
    run = [orc.sign_word(123, 77, 2, w) for w in range(1024)]
    assert run == [int(v) for v in golden["sign_run_123_77_2"]]


def test_c1_forward_bit_exact(golden):
    z = golden["c1_latent"]
    y = orc.fht_forward(z, 108618, 3, 123, 0, 108618)
    assert np.array_equal(y, golden["c1_y"])
    mid = orc.fht_forward(z, 108618, 3, 123, 1000, 2000)
    assert np.array_equal(mid, golden["c1_y_1000_2000"])
    assert np.array_equal(mid, y[1000:2000])
    # summary statistics published for this configuration
    assert y[:4] == pytest.approx([-0.50103974, 0.02545023, 0.00907144, -0.38723081], abs=1e-7)
    assert float(np.linalg.norm(y.astype(np.float64))) == pytest.approx(338.779785, rel=1e-6)


def test_c1_backward(golden):
    g = orc.fht_backward(golden["c1_grad_out"], 1024, 108618, 3, 123, 0, 108618)
    assert rel_l2(g, golden["c1_grad"]) < 1e-6
    assert float(np.linalg.norm(g.astype(np.float64))) == pytest.approx(336.063110, rel=1e-5)


@pytest.mark.parametrize("i", range(12))
def test_small_cases(golden, i):
    L, size, layers, seed, start, stop = (int(v) for v in golden["cases"][i])
    out = orc.fht_forward(golden[f"case{i}_latent"], size, layers, seed, start, stop)
    assert np.array_equal(out, golden[f"case{i}_out"])
    grad = orc.fht_backward(golden[f"case{i}_grad_out"], L, size, layers, seed, start, stop)
    ref = golden[f"case{i}_grad"]
    assert rel_l2(grad, ref) < 1e-6 or np.abs(grad - ref).max() < 1e-6


def test_fp64_mode_close_to_fp32(golden):
    z = golden["c1_latent"]
    a = orc.fht_forward(z, 108618, 3, 123, 0, 108618)
    b = orc.fht_forward(z, 108618, 3, 123, 0, 108618, precision="fp64")
    assert rel_l2(a, b) < 1e-6


def test_threads_do_not_change_results(golden):
    z = golden["c1_latent"]
    a = orc.fht_forward(z, 108618, 3, 123, 0, 108618, threads=1)
    b = orc.fht_forward(z, 108618, 3, 123, 0, 108618, threads=4)
    assert np.array_equal(a, b)


def test_linear_oracle_matches_golden(golden):
    z = golden["lin_latent"]
    w = orc.generated_weight(z, 5, 3, 2, 11)
    assert np.allclose(w, golden["lin_weight"], atol=1e-7)
    y = orc.linear_forward(golden["lin_x"], z, 3, 2, 11, bias=golden["lin_bias"])
    assert np.allclose(y, golden["lin_out"], atol=1e-6)

    z2, x2, gy = golden["lin2_latent"], golden["lin2_x"], golden["lin2_grad_y"]
    y2 = orc.linear_forward(x2, z2, 40, 3, 5, weight_scale=0.5)
    assert rel_l2(y2, golden["lin2_out"]) < 1e-6
    gx, gz, _ = orc.linear_backward(gy, x2, z2, 40, 3, 5, weight_scale=0.5)
    assert rel_l2(gx, golden["lin2_grad_x"]) < 1e-6
    assert rel_l2(gz, golden["lin2_grad_latent"]) < 1e-5


def test_invalid_slice_rejected():
    with pytest.raises(ValueError):
        orc.fht_forward(np.ones(4, np.float32), 10, 1, 0, 5, 11)
