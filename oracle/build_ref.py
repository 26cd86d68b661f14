"""Build recipe for oracle/_ref/: the reference's own gt_flash_attention compiled from its source --
TEST INFRASTRUCTURE ONLY (a checker for the CPU restatement, never the product path).

The reference's native library cannot be built here as a whole (csrc/gt_internal.h includes ggml
headers from a llama.cpp tree that build_native.py downloads, build_native.py:217-307). Its SDPA
forward, gt_flash_attention (csrc/gt_ops_nn.cpp:2423-2525), is a self-contained host loop that uses
none of ggml. This recipe reads that one function out of the reference's source file where it lies
(found by its signature, ended by brace matching), writes it with oracle/ref_shim.h in front into
oracle/_ref/ (git-ignored; nothing from the reference is committed), adds a plain-array C wrapper
and compiles it with the reference's own flags (-O3 -fopenmp, build_native.py:564-586).

The built library travels with the tree; the reference source is needed only to build it.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
LIB = OUT / "libgt_ref_attn.so"
SHIM = HERE / "ref_shim.h"
REF_SRC = Path(os.environ.get("GT_REFERENCE_ROOT", "/root/reference")) / "csrc" / "gt_ops_nn.cpp"
SIGNATURE = 'extern "C" gt_tensor * gt_flash_attention('

WRAPPER = r"""
// plain-array entry point of the reference function above (written for this checker)
extern "C" const char* ref_last_error() { return shim_error().c_str(); }

static gt_tensor view4(const void* p, int dt, int nd, const int64_t* s) {
    gt_tensor t;
    t.ndim = nd;
    t.dtype = dt;
    t.numel = 1;
    for (int i = nd - 1; i >= 0; --i) {
        t.shape[i] = s[i];
        t.strides[i] = t.numel;
        t.numel *= s[i];
    }
    t.data = const_cast<void*>(p);
    return t;
}

extern "C" int ref_flash_attention(const void* q, const void* k, const void* v, int dtype, int64_t B, int64_t H,
                                   int64_t L, int64_t D, int64_t Hkv, int64_t S, int64_t Dv, const void* mask,
                                   int mask_dtype, int mask_ndim, const int64_t* mask_shape, float scale,
                                   int is_causal, void* out) {
    const int64_t qs[4] = {B, H, L, D}, ks[4] = {B, Hkv, S, D}, vs[4] = {B, Hkv, S, Dv};
    gt_tensor tq = view4(q, dtype, 4, qs), tk = view4(k, dtype, 4, ks), tv = view4(v, dtype, 4, vs);
    gt_tensor tm;
    if (mask) tm = view4(mask, mask_dtype, mask_ndim, mask_shape);
    gt_tensor* o = gt_flash_attention(&tq, &tk, &tv, mask ? &tm : nullptr, scale, is_causal);
    if (!o) return -1;
    std::memcpy(out, o->data, (size_t)o->numel * shim_elem_size(o->dtype));
    gt_tensor_free(o);
    return 0;
}
"""


def extract_function(text: str) -> str:
    """The text of gt_flash_attention in the reference source: from its signature to the brace
    that closes its body."""
    start = text.find(SIGNATURE)
    if start < 0:
        raise RuntimeError("gt_flash_attention not found in the reference source")
    depth, i, opened = 0, text.index("{", start), False
    while i < len(text):
        c = text[i]
        if c == "{":
            depth += 1
            opened = True
        elif c == "}":
            depth -= 1
            if opened and depth == 0:
                return text[start:i + 1]
        i += 1
    raise RuntimeError("unbalanced braces in gt_flash_attention")


def available() -> bool:
    return LIB.exists() or REF_SRC.exists()


def build(force: bool = False, verbose: bool = False) -> Path | None:
    """Build oracle/_ref/libgt_ref_attn.so when the reference source is present; returns the library
    path (an already-built library is reused, e.g. on a machine without the reference), or None."""
    if LIB.exists() and not force and (not REF_SRC.exists() or LIB.stat().st_mtime >= SHIM.stat().st_mtime):
        return LIB
    if not REF_SRC.exists():
        return LIB if LIB.exists() else None
    OUT.mkdir(exist_ok=True)
    body = extract_function(REF_SRC.read_text())
    src = OUT / "gt_flash_attention_ref.cpp"
    src.write_text(f'#include "{SHIM}"\n\n// {REF_SRC} (gt_flash_attention)\n' + body + "\n" + WRAPPER)
    cxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"
    cmd = [cxx, "-O3", "-march=x86-64-v3", "-fopenmp", "-std=c++17", "-shared", "-fPIC", str(src), "-o",
           str(LIB) + ".tmp"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    try:
        subprocess.run(cmd, check=True)
    finally:
        src.unlink()  # the extracted reference text is not kept beside the library
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
