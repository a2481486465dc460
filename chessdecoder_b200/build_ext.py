"""Builds libcdk.so (the sm_100a kernel library) in-tree with nvcc.

Each ``csrc/*.cu`` file compiles to a relocatable object in parallel
(``-rdc=true``, because the device error word is shared across files), then
one device-link step and one host link produce
``chessdecoder_b200/libcdk.so``.  Objects are rebuilt only when a source or
header is newer than them.

Usage: ``python -m chessdecoder_b200.build_ext [--force] [--verbose]``
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
BUILD = ROOT / "_build"
LIB = PKG / "libcdk.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-rdc=true",
              "--expt-relaxed-constexpr", "-Xptxas", "-v" if os.environ.get("CDK_PTXAS_VERBOSE") else "-O3"]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; libcdk.so needs the CUDA 12.9 toolchain")
    return cand


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _compile(nvcc: str, src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if os.environ.get("CDK_PTXAS_VERBOSE"):
        sys.stdout.write(res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    nvcc = nvcc_path()
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    newest_hdr = max((h.stat().st_mtime for h in _headers()), default=0.0)
    todo = []
    for s in srcs:
        obj = BUILD / (s.stem + ".o")
        if force or not obj.exists() or obj.stat().st_mtime < max(s.stat().st_mtime, newest_hdr):
            todo.append(s)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            list(ex.map(lambda s: _compile(nvcc, s, verbose), todo))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        dlink = BUILD / "dlink.o"
        cmd = [nvcc, *ARCH, "-Xcompiler", "-fPIC", "-dlink", *map(str, objs), "-o", str(dlink)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), str(dlink), "-o", str(tmp),
               "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
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
