"""Build libmlxp_attn.so in-tree for sm_100a with nvcc (no torch extension machinery).

    python mlx-primitives_b200/csrc/build.py [--force] [--debug]

The library lands next to the Python package (mlx_primitives/libmlxp_attn.so) so that it
travels with the source tree; the Python shim loads it from there (or from $MLXP_LIB).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG_ROOT = CSRC.parent
INCLUDE = PKG_ROOT.parent / "include"
OUT = PKG_ROOT / "mlx_primitives" / "libmlxp_attn.so"
SOURCES = [CSRC / "mlxp_attn.cu"]
DEPS = SOURCES + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "mlxp_attn.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set $NVCC)")


def command(debug: bool = False, verbose_ptxas: bool = False) -> list[str]:
    cmd = [nvcc_path(), *ARCH, "-std=c++17", "-O3", "-lineinfo", "-shared",
           "-Xcompiler", "-fPIC", "-cudart", "shared",
           "-Xlinker", "-rpath,/usr/local/cuda/lib64",
           "-I", str(INCLUDE), "-o", str(OUT), "-ldl"]
    if debug:
        cmd += ["-DMLXP_DEBUG_CHECKS=1"]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    cmd += [str(s) for s in SOURCES]
    return cmd


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in DEPS if d.exists())


def build(force: bool = False, debug: bool = False, verbose_ptxas: bool = False) -> Path:
    if not force and not debug and not verbose_ptxas and up_to_date():
        return OUT
    cmd = command(debug=debug, verbose_ptxas=verbose_ptxas)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose_ptxas:
        sys.stderr.write(res.stderr)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, debug=a.debug, verbose_ptxas=a.ptxas_v))
