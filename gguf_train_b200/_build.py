"""Build of the engine's native library (sm_100a only).

Compiles gguf_train_b200/csrc/*.cu and *.cpp with nvcc for `-gencode arch=compute_100a,code=sm_100a`
and links them into gguf_train_b200/_lib/libgt_attn_b200.so, in-tree, so the built library travels
with the source tree. The CUDA runtime is linked statically, so the library needs only the NVIDIA
driver at run time. Objects are rebuilt when a source or header is newer than the library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIBDIR = PKG / "_lib"
OBJDIR = PKG / "_build"
LIB = LIBDIR / "libgt_attn_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", str(INCLUDE)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the B200 engine cannot be built")


def _sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers():
    return sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> Path:
    """Compile every CUDA/C++ source for sm_100a and link the shared library. Returns its path."""
    srcs = _sources()
    hdrs = _headers()
    if not force and not _stale(LIB, srcs + hdrs + [Path(__file__)]):
        return LIB
    LIBDIR.mkdir(exist_ok=True)
    OBJDIR.mkdir(exist_ok=True)
    cc = nvcc()
    flags = NVCC_FLAGS + list(extra_flags or [])

    def compile_one(src: Path) -> Path:
        obj = OBJDIR / (src.name + ".o")
        if force or _stale(obj, [src] + hdrs + [Path(__file__)]):
            cmd = [cc] + ARCH + flags + ["-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
            if verbose and (r.stdout or r.stderr):
                print(r.stdout + r.stderr, file=sys.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc] + ARCH + ["-shared", "-cudart", "static", "-o", str(tmp)] + [str(o) for o in objs] + ["-ldl", "-lpthread", "-lrt"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
