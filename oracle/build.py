"""Build recipe for the CPU oracle (test infrastructure, not product code).

Compiles oracle/sdpa_oracle.cpp into oracle/liboracle_sdpa.so with the flags the reference uses
for its native build (build_native.py:564-586: -O3 -fopenmp), except that -march is pinned to
x86-64-v3 instead of "native": the library is built on one host and run on another.

The reference's native library as a whole cannot be compiled here (gt_ops_nn.cpp includes
gt_internal.h, which needs ggml headers from a llama.cpp tree that build_native.py downloads,
build_native.py:217-307). Its SDPA forward, gt_flash_attention, needs none of ggml: oracle/build_ref.py
compiles that one function from the reference source into oracle/_ref/, and tests pin this
restatement to it.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "sdpa_oracle.cpp"
LIB = HERE / "liboracle_sdpa.so"


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    # the system g++ ships libgomp; a CXX from the environment may not
    cxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"
    cmd = [cxx, "-O3", "-march=x86-64-v3", "-fopenmp", "-std=c++17", "-shared", "-fPIC",
           str(SRC), "-o", str(LIB) + ".tmp"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
