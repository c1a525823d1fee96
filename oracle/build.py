"""Build recipe for the CPU oracle (TEST INFRASTRUCTURE ONLY).

Two shared libraries:

* ``oracle/_build/liboracle.so`` -- this repository's C restatement (``apex_oracle.c``).
* ``oracle/_ref/libapexref.so`` -- the reference's OWN CPU code for the path, compiled from
  the reference tree where it lies: ``src/tests/cpu_ref.h`` (with its ``../nvfp4.h``
  include) and the ``ropeCpu`` / ``attentionRowCpu`` code block of
  ``docs/B6_3_attention.md`` section 5, which is written unchanged into
  ``oracle/_ref/doc_cpu_ref_additions.h`` at build time.  Built only when the reference tree
  is present; the result is git-ignored and travels with the working tree.

The reference tree is ``--reference DIR``, else ``$APEX_REFERENCE_DIR``, else a checkout named
``reference`` beside this repository's directory.

Usage: ``python oracle/build.py [--reference DIR]``.
"""
from __future__ import annotations

import argparse
import os
import pathlib
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"
# a reference checkout beside this repository (overridden by --reference / $APEX_REFERENCE_DIR)
SIBLING_REFERENCE_DIR = HERE.parent.parent / "reference"

ORACLE_LIB = BUILD / "liboracle.so"
REF_LIB = REF_OUT / "libapexref.so"

_DOC_HEADING = "## 5. `cpu_ref.h` additions"


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def build_oracle() -> pathlib.Path:
    BUILD.mkdir(exist_ok=True)
    src = HERE / "apex_oracle.c"
    if ORACLE_LIB.exists() and ORACLE_LIB.stat().st_mtime >= src.stat().st_mtime:
        return ORACLE_LIB
    _run(["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
          "-o", str(ORACLE_LIB), str(src), "-lm"])
    return ORACLE_LIB


def extract_doc_block(doc_path: pathlib.Path) -> str:
    """Return the first ```cpp block after the section-5 heading of the design doc."""
    text = doc_path.read_text()
    at = text.find(_DOC_HEADING)
    if at < 0:
        raise RuntimeError(f"{doc_path}: section heading not found")
    start = text.find("```cpp", at)
    end = text.find("```", start + 6)
    if start < 0 or end < 0:
        raise RuntimeError(f"{doc_path}: code block not found")
    return text[start + len("```cpp"):end]


def build_reference(reference_dir: str | os.PathLike | None = None) -> pathlib.Path | None:
    ref = pathlib.Path(reference_dir or os.environ.get("APEX_REFERENCE_DIR") or SIBLING_REFERENCE_DIR)
    cpu_ref = ref / "src" / "tests" / "cpu_ref.h"
    doc = ref / "docs" / "B6_3_attention.md"
    if not (cpu_ref.exists() and doc.exists()):
        return REF_LIB if REF_LIB.exists() else None
    REF_OUT.mkdir(exist_ok=True)
    header = REF_OUT / "doc_cpu_ref_additions.h"
    header.write_text(
        "// Generated at build time from docs/B6_3_attention.md section 5 (reference tree).\n"
        "#pragma once\n#include <algorithm>\n#include <cmath>\n#include <cstddef>\n"
        "#include <cstdint>\n#include <vector>\n" + extract_doc_block(doc))
    _run(["g++", "-O2", "-std=c++20", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
          "-I", str(cpu_ref.parent), "-I", str(REF_OUT),
          "-o", str(REF_LIB), str(HERE / "ref_shim.cpp")])
    return REF_LIB


def main(argv: list[str]) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    args = ap.parse_args(argv)
    print("oracle:", build_oracle())
    print("reference:", build_reference(args.reference))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
