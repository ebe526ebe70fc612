"""Generate ``golden_fht_mix.npz`` from the reference's FixedFHTMix.

Usage:  python tests/golden/make_golden_mix.py <path-to-reference-checkout>

Imports ``examples.nanogpt.model`` from the given checkout and records, per
case, the module's sign buffer, a seeded input, its output and the input
gradient of sum(y * g) (pure torch, CPU, fp32).  The reference is needed
only to regenerate this file, not to run the tests.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "golden_fht_mix.npz"

# (features, seed, rows)
CASES = [(1, 3, 2), (24, 5, 3), (96, 11, 4), (768, 66, 5), (1600, 130, 3), (3072, 98, 2), (6400, 7, 2)]


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import examples.nanogpt.model as ref_model

    data = {}
    for i, (features, seed, rows) in enumerate(CASES):
        mix = ref_model.FixedFHTMix(features, seed)
        g = torch.Generator().manual_seed(1000 + i)
        x = torch.randn(rows, features, generator=g, requires_grad=True)
        gy = torch.randn(rows, features, generator=g)
        y = mix(x)
        (y * gy).sum().backward()
        data[f"mix{i}_meta"] = np.array([features, seed, rows], dtype=np.int64)
        data[f"mix{i}_signs"] = mix.signs.numpy().astype(np.float32)
        data[f"mix{i}_x"] = x.detach().numpy()
        data[f"mix{i}_g"] = gy.numpy()
        data[f"mix{i}_y"] = y.detach().numpy()
        data[f"mix{i}_gx"] = x.grad.numpy()
    data["count"] = np.array(len(CASES), dtype=np.int64)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({len(CASES)} cases)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../reference")
