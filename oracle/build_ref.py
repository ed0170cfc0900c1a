"""Compile the reference's scalar kernel baselines into oracle/_ref/.

TEST INFRASTRUCTURE. Each kernels/<k>/baseline.c of the reference (hexlib)
is the "correct and obvious, never fast" C statement of one kernel, with
fp32 arithmetic and one rounding per output. They need nothing but their own
kernel_api.h and libm, so they are compiled here with the host gcc, straight
from the reference checkout (read-only), with `__fp16` spelled `_Float16`
(the host compiler's IEEE half type). The output, oracle/_ref/libhexref.so,
is a build artefact: it is git-ignored but travels with the tree, so the
GPU-side tests and the CPU-baseline timing can call the reference's own
arithmetic where the reference itself is absent.

Usage: python oracle/build_ref.py /path/to/hexlib-checkout
       (or HEXLIB_REFERENCE=/path/to/hexlib-checkout python oracle/build_ref.py)
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libhexref.so")

# kernel directory -> its baseline symbol; hmx_matmul_fp16 has no encoder op
KERNELS = {
    "add_fp16": "add_fp16_baseline",
    "cast_f32_f16": "cast_f32_f16_baseline",
    "layernorm_fp16": "layernorm_fp16_baseline",
    "matmul_fp16": "matmul_fp16_baseline",
    "matmul_epilogue_fp16": "matmul_epilogue_fp16_baseline",
    "patchify_fp32": "patchify_fp32_baseline",
    "rmsnorm_fp16": "rmsnorm_fp16_baseline",
    "rope_2d_fp16": "rope_2d_fp16_baseline",
    "scale_fp16": "scale_fp16_baseline",
    "softmax_fp16": "softmax_fp16_baseline",
    "transpose_hd_fp16": "transpose_hd_fp16_baseline",
    "transpose_th_fp16": "transpose_th_fp16_baseline",
}


def build(ref_root: str | None) -> str | None:
    """Build libhexref.so from the reference checkout at `ref_root`; return its
    path (an existing prebuilt one is returned when no checkout is given or
    it is absent, as on a GPU box that only runs the prebuilt file)."""
    if not ref_root:
        return LIB if os.path.exists(LIB) else None
    kdir = os.path.join(ref_root, "kernels")
    if not os.path.isdir(kdir):
        return LIB if os.path.exists(LIB) else None
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no host C compiler")
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = os.path.join(OUT_DIR, "obj")
    os.makedirs(tmp, exist_ok=True)
    objs = []
    for k in KERNELS:
        src = os.path.join(kdir, k, "baseline.c")
        obj = os.path.join(tmp, f"{k}.o")
        if not os.path.exists(obj) or os.path.getmtime(obj) < os.path.getmtime(src):
            cmd = [cc, "-O2", "-fPIC", "-std=gnu11", "-D__fp16=_Float16",
                   "-I", os.path.join(kdir, k), "-c", src, "-o", obj]
            subprocess.run(cmd, check=True, capture_output=True, text=True)
        objs.append(obj)
    if not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        subprocess.run([cc, "-shared", "-o", LIB, *objs, "-lm"], check=True,
                       capture_output=True, text=True)
    return LIB


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HEXLIB_REFERENCE")
    if not root:
        sys.exit("usage: python oracle/build_ref.py /path/to/hexlib-checkout "
                 "(or set HEXLIB_REFERENCE)")
    print(build(root))
