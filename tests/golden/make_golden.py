"""Generate the golden fixtures in this folder from the reference implementation.

Usage:  python tests/golden/make_golden.py <path-to-reference-checkout>

The reference package ``latent_weight_lab`` is imported from the given
checkout (its pure-torch CPU path, ``block_fht_slice_torch`` and autograd),
and its outputs are written to ``golden_block_fht.npz``.  The fixtures pin
the CPU oracle (oracle/) and, through it, the CUDA path.  The reference is
not needed to run the tests; only to regenerate these files.
"""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "golden_block_fht.npz"

# (seed, block, layer, word) points for the bit-exact sign-word table.
SIGN_POINTS = [
    (0, 0, 0, 0), (123, 0, 0, 0), (123, 106, 3, 31), (999, 3, 2, 4),
    (2**40 + 5, 8191, 2, 1023), (-1, 1, 1, 1), (7, 0, 1, 0), (2**63 - 1, 5, 3, 7),
    (-(2**63), 2, 0, 9), (123, 8191, 3, 1023), (0xDEADBEEF, 12345, 1, 262143),
    (1 << 32, 0, 0, 0), (5, 1 << 20, 2, 3),
]

# (latent_size, size, layers, seed, start, stop)  -- small forward/backward cases
CASES = [
    (1, 5, 1, 3, 0, 5),
    (7, 31, 2, 123, 3, 17),
    (8, 40, 2, 7, 5, 23),
    (31, 100, 3, 11, 0, 100),
    (32, 64, 1, 1, 0, 64),
    (33, 200, 3, -1, 17, 199),
    (100, 1000, 2, 2**40 + 5, 250, 777),
    (1000, 5000, 3, 42, 0, 5000),
    (4096, 8192, 1, 123, 17, 4099),
    (20000, 65536, 1, 123, 111, 4096),
    (4096, 20000, 3, 9, 0, 20000),
    (300, 2048, 3, 77, 512, 512),   # empty slice
]


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    bf = importlib.import_module("latent_weight_lab.block_fht")
    data: dict[str, np.ndarray] = {}

    data["sign_points"] = np.array(SIGN_POINTS, dtype=object).astype(str)
    data["sign_words"] = np.array([bf.sign_word_for(*p) for p in SIGN_POINTS], dtype=np.uint64)
    # a run of consecutive words for vectorised checks
    run = np.array([bf.sign_word_for(123, 77, 2, w) for w in range(1024)], dtype=np.uint64)
    data["sign_run_123_77_2"] = run

    # Config C1: BlockFHT(latent[1024], size=108618, layers=3, seed=123)
    torch.manual_seed(0)
    z = torch.randn(1024)
    torch.manual_seed(1)
    g = torch.randn(108618)
    zz = z.clone().requires_grad_(True)
    y = bf.block_fht_slice_torch(zz, 108618, 3, 123, 0, 108618)
    (y * g).sum().backward()
    y_mid = bf.block_fht_slice_torch(z, 108618, 3, 123, 1000, 2000)
    data["c1_latent"] = z.numpy()
    data["c1_y"] = y.detach().numpy()
    data["c1_y_1000_2000"] = y_mid.numpy()
    data["c1_grad_out"] = g.numpy()
    data["c1_grad"] = zz.grad.numpy()

    # Small cases with a seeded latent and grad_out
    for i, (L, size, layers, seed, start, stop) in enumerate(CASES):
        torch.manual_seed(100 + i)
        z = torch.randn(L)
        go = torch.randn(stop - start)
        zz = z.clone().requires_grad_(True)
        out = bf.block_fht_slice_torch(zz, size, layers, seed, start, stop)
        if out.numel():
            (out * go).sum().backward()
            grad = zz.grad.numpy()
        else:
            grad = np.zeros(L, dtype=np.float32)
        data[f"case{i}_latent"] = z.numpy()
        data[f"case{i}_grad_out"] = go.numpy()
        data[f"case{i}_out"] = out.detach().numpy()
        data[f"case{i}_grad"] = grad
    data["cases"] = np.array(CASES, dtype=np.int64)

    # The reference bf16 path (every stage rounded to bf16), for reporting only.
    torch.manual_seed(5)
    zb = torch.randn(4096).to(torch.bfloat16)
    yb = bf.block_fht_slice_torch(zb, 16384, 3, 123, 0, 16384)
    data["bf16_latent_as_f32"] = zb.float().numpy()
    data["bf16_ref_out_as_f32"] = yb.float().numpy()

    # BlockFHTLinear forward / backward (block_fht.py:291-356)
    torch.manual_seed(123)
    layer = bf.BlockFHTLinear(5, 3, bias=True, latent_dim=8, layers=2, seed=11)
    x = torch.randn(4, 5)
    out = layer(x)
    out.square().mean().backward()
    data["lin_latent"] = layer.generator.latent.detach().numpy()
    data["lin_bias"] = layer.bias.detach().numpy()
    data["lin_x"] = x.numpy()
    data["lin_weight"] = layer.weight.detach().numpy()
    data["lin_out"] = out.detach().numpy()
    data["lin_grad_latent"] = layer.generator.latent.grad.numpy()
    data["lin_grad_bias"] = layer.bias.grad.numpy()

    torch.manual_seed(7)
    layer2 = bf.BlockFHTLinear(96, 40, bias=False, latent_dim=300, layers=3, seed=5, weight_scale=0.5)
    x2 = torch.randn(6, 96, requires_grad=True)
    out2 = layer2(x2)
    torch.manual_seed(8)
    gy = torch.randn_like(out2)
    (out2 * gy).sum().backward()
    data["lin2_latent"] = layer2.generator.latent.detach().numpy()
    data["lin2_x"] = x2.detach().numpy()
    data["lin2_out"] = out2.detach().numpy()
    data["lin2_grad_y"] = gy.numpy()
    data["lin2_grad_x"] = x2.grad.numpy()
    data["lin2_grad_latent"] = layer2.generator.latent.grad.numpy()

    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(data)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(sys.argv[1])
