"""Builds libfuton_cuda.so (sm_100a) in-tree with nvcc.

Each translation unit under csrc/ compiles in parallel; the objects link into
futon_b200/libfuton_cuda.so with the CUDA runtime linked statically, so the
library only needs the NVIDIA driver at run time. The tokenizer's Unicode
tables (unicode_tables.h) are generated into the build folder first by
csrc/gen_unicode_tables.py. Usage:
    python -m futon_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libfuton_cuda.so"
SOURCES = ["futon_cuda.cu", "gemm_f16.cu", "gemm_bf16.cu", "gemm_s8.cu", "tokenizer.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libfuton_cuda")


def _deps() -> list[Path]:
    return (sorted(CSRC.glob("*.cu*")) + sorted(CSRC.glob("*.cpp")) + sorted(CSRC.glob("*.py"))
            + sorted((ROOT / "include").glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    deps = _deps()
    if not force and not _stale(LIB, deps):
        return LIB
    BUILD.mkdir(exist_ok=True)
    r = subprocess.run([sys.executable, str(CSRC / "gen_unicode_tables.py"),
                        str(BUILD / "unicode_tables.h")], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"gen_unicode_tables.py failed:\n{r.stdout}\n{r.stderr}")
    cc = nvcc()
    common = ARCH + [
        "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
        "-I", str(ROOT / "include"), "-I", str(CSRC), "-I", str(BUILD),
    ]
    if verbose:
        common += ["-Xptxas", "-v"]

    def compile_one(src: str) -> Path:
        obj = BUILD / (Path(src).stem + ".o")
        cmd = [cc, *common, "-c", str(CSRC / src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr:
            sys.stderr.write(r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
