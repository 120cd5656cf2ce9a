"""TEST INFRASTRUCTURE ONLY: build oracle/_ref/libg16ref_gpu.so from the reference's own kernels.

The reference (gtx16_fp16) keeps its CUDA C kernels as one string, _SRC, in
src/gtx16_fp16/kernels.py:19-251, and compiles it at run time with NVRTC using
["--use_fast_math", "-std=c++17"] (kernels.py:352-353). This script reads that string from the
read-only reference checkout, writes it to a temporary directory, compiles it together with
oracle/ref_launch.cu (launchers restating the reference's host dispatch) with the same options for
sm_100a, and deletes the temporary copy. Only the built library is kept, under oracle/_ref/ (ignored
by git). The GPU box never reads the reference checkout; it loads the prebuilt library.

Usage: python oracle/build_ref.py --reference <reference checkout>
       (or set G16_REFERENCE_DIR; there is no default location)
"""
from __future__ import annotations

import argparse
import ast
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
OUT = os.path.join(OUT_DIR, "libg16ref_gpu.so")
ENV_VAR = "G16_REFERENCE_DIR"


def reference_dir(explicit: str | None = None) -> str | None:
    """The reference checkout: `explicit`, else $G16_REFERENCE_DIR, else None."""
    return explicit or os.environ.get(ENV_VAR) or None


def extract_src(kernels_py: str) -> str:
    """Value of the module-level string assignment `_SRC = r\"\"\"...\"\"\"` (parsed, not executed)."""
    tree = ast.parse(open(kernels_py).read())
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id == "_SRC" for t in node.targets):
            if isinstance(node.value, ast.Constant) and isinstance(node.value.value, str):
                return node.value.value
    raise RuntimeError(f"_SRC string not found in {kernels_py}")


def build(reference: str | None = None, quiet: bool = False) -> str | None:
    reference = reference_dir(reference)
    kernels_py = os.path.join(reference, "src", "gtx16_fp16", "kernels.py") if reference else ""
    if not kernels_py or not os.path.exists(kernels_py):
        if not quiet:
            print(f"build_ref: no reference checkout ({kernels_py or 'none given'}); skipping "
                  f"(prebuilt {OUT} is used if present)")
        return OUT if os.path.exists(OUT) else None
    src = extract_src(kernels_py)
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = tempfile.mkdtemp(prefix="g16ref_")
    try:
        kpath = os.path.join(tmp, "reference_kernels.cuh")
        with open(kpath, "w") as f:
            f.write(src)
        cmd = ["nvcc", "-O3", "--use_fast_math", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
               "-shared", "-Xcompiler", "-fPIC", f'-DREF_KERNELS="{kpath}"', "-o", OUT,
               os.path.join(HERE, "ref_launch.cu")]
        subprocess.run(cmd, check=True)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help=f"reference checkout (else ${ENV_VAR})")
    a = ap.parse_args()
    if reference_dir(a.reference) is None:
        ap.error(f"give --reference or set {ENV_VAR}")
    out = build(a.reference)
    print(out or "not built")
    sys.exit(0)
