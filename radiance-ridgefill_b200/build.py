"""Build the B200 RidgeFill kernel library in-tree: radiance-ridgefill_b200/ridgefill.so.

    python radiance-ridgefill_b200/build.py [--force] [--verbose]

Every CUDA source is compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``) with
``-lineinfo``; the host sources (operand parsing, the row table) go through the same nvcc link. The
CUDA runtime is linked statically, so the library loads wherever the driver does. The library has no
host rows and no CPU fallback: every row launches CUDA work.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
OUT = HERE / "ridgefill.so"
BUILD = HERE / "_build"

CUDA_SOURCES = ["small_ops.cu", "mask.cu", "gemm_q.cu", "gdn.cu", "conv_prep.cu", "attn_kv.cu", "peer.cu"]
HOST_SOURCES = ["parse.cpp", "rows.cpp", "folder.cpp"]
HEADERS = ["common.cuh", "sm100.cuh", "mma.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the B200 library needs the CUDA toolkit to build")


def host_cxx() -> str:
    return "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"


def _inputs() -> list[Path]:
    inc = ROOT / "include"
    return ([CSRC / s for s in CUDA_SOURCES + HOST_SOURCES + HEADERS] +
            [inc / h for h in ("rad_abi.h", "rad_plugin.h", "ridgefill.h", "ridgefill_schemas.h", "ridgefill_folder.h", "ridgefill_team.h")] + [Path(__file__)])


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    common = ["-std=c++17", "-O3", "-Xcompiler", "-fPIC", f"-I{ROOT / 'include'}", f"-I{CSRC}",
              "-ccbin", host_cxx()]
    objs = []
    for src in CUDA_SOURCES:
        obj = BUILD / (src + ".o")
        cmd = [cc, *ARCH, "-lineinfo", *common, "-Xptxas", "-v" if verbose else "-O3", "-c", str(CSRC / src),
               "-o", str(obj)]
        _run(cmd, verbose)
        objs.append(obj)
    for src in HOST_SOURCES:
        obj = BUILD / (src + ".o")
        _run([cc, *common, "-c", str(CSRC / src), "-o", str(obj)], verbose)
        objs.append(obj)
    tmp = OUT.with_suffix(".so.tmp")
    _run([cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs), "-ldl", "-lpthread", "-lrt"],
         verbose)
    tmp.replace(OUT)
    return OUT


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:2])} ... {cmd[-3]}")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
