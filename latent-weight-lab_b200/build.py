"""Build liblwl_b200.so (the sm_100a BlockFHT library) in-tree with nvcc.

    python latent-weight-lab_b200/build.py [--force] [--verbose]

Output: latent-weight-lab_b200/latent_weight_lab/_lib/liblwl_b200.so.  Each
.cu file is compiled to an object under _build/ (skipped when up to date),
then linked against the shared CUDA runtime so the library shares torch's
runtime when both live in one process.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
BUILD_DIR = PKG_ROOT / "_build"
LIB_DIR = PKG_ROOT / "latent_weight_lab" / "_lib"
LIB = LIB_DIR / "liblwl_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda) / "bin" / "nvcc"
    return str(cand) if cand.exists() else (shutil.which("nvcc") or "nvcc")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def build(force: bool = False, verbose: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    hdr_mtime = max((h.stat().st_mtime for h in _headers()), default=0.0)
    objs, cmds = [], []
    changed = force or not LIB.exists()
    for src in sorted(CSRC.glob("*.cu")):
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_mtime):
            cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd += ["-Xptxas", "-v"]
                print(" ".join(cmd), flush=True)
            cmds.append(cmd)
    if cmds:
        # translation units compile independently: one nvcc per file, in parallel
        with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as pool:
            for _ in pool.map(lambda c: subprocess.run(c, check=True), cmds):
                pass
        changed = True
    if changed or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cuda = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "shared", "-o", str(LIB), *map(str, objs),
               "-lcublas", "-Xlinker", f"-rpath,{cuda / 'lib64'}"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    sys.exit(0)
