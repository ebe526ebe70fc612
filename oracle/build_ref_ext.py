"""Builds the reference's own CUDA extension (test infrastructure, not product code).

Compiles the reference sources where they lie -- csrc/block_fht_ext.cpp and
csrc/block_fht_ext_cuda.cu of the reference checkout -- with torch's extension
builder, the flags the reference itself passes (latent_weight_lab/block_fht.py:
132-140: -O3, --use_fast_math) plus code for sm_100a, into oracle/_ref/.  The
module it produces (lwl_ref_block_fht_ext) is the reference's fp32 GPU
transform and fused linear; tests/test_reference_ext_gpu.py loads it to check
the library against the reference's own CUDA kernels and to time both on the
same B200.  Nothing in the product imports it.

    python oracle/build_ref_ext.py [--reference PATH]
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "lwl_ref_block_fht_ext"


def build(reference: Path) -> Path | None:
    srcs = [reference / "csrc" / "block_fht_ext.cpp", reference / "csrc" / "block_fht_ext_cuda.cu"]
    if not all(p.exists() for p in srcs):
        return None
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    try:
        import ninja

        os.environ["PATH"] = f"{ninja.BIN_DIR}:" + os.environ.get("PATH", "")
    except Exception:  # noqa: BLE001
        pass
    from torch.utils.cpp_extension import load

    OUT.mkdir(exist_ok=True)
    load(name=NAME, sources=[str(p) for p in srcs], build_directory=str(OUT),
         extra_cuda_cflags=["-O3", "--use_fast_math", "-gencode", "arch=compute_100a,code=sm_100a"],
         extra_cflags=["-O3"], verbose=False)
    so = next(OUT.glob(f"{NAME}*.so"), None)
    return so


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("LWL_REFERENCE", "/root/reference"))
    args = ap.parse_args()
    so = build(Path(args.reference))
    print(so if so else "reference sources not found; nothing built")
    sys.exit(0)
