"""Builds and runs the C++ harness tests/cpp/test_backend.cpp: CudaBackend + ops.h (the
reference's Backend / ops interface) against the oracle, on the GPU."""
from __future__ import annotations

import pathlib
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def build_harness() -> pathlib.Path:
    from apex_b200 import build as nbuild
    from oracle import build as obuild
    lib = nbuild.build()
    olib = obuild.build_oracle()
    exe = ROOT / "tests" / "cpp" / "_build" / "test_backend"
    exe.parent.mkdir(exist_ok=True)
    src = ROOT / "tests" / "cpp" / "test_backend.cpp"
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", str(ROOT / "apex_b200" / "csrc"), "-I", str(ROOT / "include"),
                    "-I", "/usr/local/cuda/include", str(src), "-o", str(exe),
                    "-L", str(lib.parent), "-lapex_cuda", f"-Wl,-rpath,{lib.parent}",
                    "-L", str(olib.parent), "-loracle", f"-Wl,-rpath,{olib.parent}"], check=True)
    return exe


def test_cpp_backend_harness():
    exe = build_harness()
    proc = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    print(proc.stdout)
    assert proc.returncode == 0, proc.stdout + proc.stderr
