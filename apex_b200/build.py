"""Build the in-tree native library and CLI of apex_b200 for sm_100a.

Outputs (git-ignored, shipped with the working tree):
  apex_b200/lib/libapex_cuda.so   C ABI of include/apex_cuda.h (kernels + entry points) and the
                                  C++ CudaBackend (csrc/backend/cuda) behind the reference's
                                  apex::Backend interface
  apex_b200/lib/apex_cuda_cli     the reference-style command-line harness (test-attn etc.)

Every .cu is compiled with ``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``.
Usage: python -m apex_b200.build [--verbose]  (``-Xptxas -v`` register report with --verbose)
"""
from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
OBJ_DIR = PKG / "lib" / "obj"
LIB = LIB_DIR / "libapex_cuda.so"
CLI = LIB_DIR / "apex_cuda_cli"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", str(ROOT / "include")]

KERNEL_SOURCES = sorted((CSRC / "kernels").glob("*.cu"))
BACKEND_SOURCES = sorted((CSRC / "backend" / "cuda").glob("*.cpp")) + sorted((CSRC / "loader").glob("*.cpp"))
CLI_SOURCES = [CSRC / "main.cpp"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _run(cmd, verbose=False):
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout + proc.stderr)
    if proc.returncode != 0:
        raise RuntimeError("build failed: " + " ".join(map(str, cmd)) + "\n" + proc.stdout + proc.stderr)
    return proc


def _stale(target: pathlib.Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(pathlib.Path(d).stat().st_mtime > t for d in deps)


def _headers():
    return (list((CSRC).rglob("*.h")) + list((CSRC).rglob("*.cuh")) + list((ROOT / "include").glob("*.h")))


def build(verbose: bool = False, force: bool = False) -> pathlib.Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    objs = []
    for src in KERNEL_SOURCES + BACKEND_SOURCES:
        obj = OBJ_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            extra = ["-Xptxas", "-v"] if (verbose and src.suffix == ".cu") else []
            lang = [] if src.suffix == ".cu" else ["-x", "cu"]
            _run([nvcc(), *ARCH, *NVCC_FLAGS, *extra, *lang, "-c", str(src), "-o", str(obj)], verbose)
    if force or _stale(LIB, objs):
        _run([nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcuda"], verbose)
    cli_srcs = [s for s in CLI_SOURCES if s.exists()]
    if cli_srcs and (force or _stale(CLI, cli_srcs + headers + [LIB])):
        _run([nvcc(), *ARCH, *NVCC_FLAGS, "-x", "cu", *map(str, cli_srcs), "-o", str(CLI),
              "-L", str(LIB_DIR), "-lapex_cuda", "-Xlinker", "-rpath=$ORIGIN"], verbose)
    return LIB


def main(argv):
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    print(build(verbose=args.verbose, force=args.force))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
