"""Build libhexlib_b200.so in-tree, for sm_100a only.

Each `csrc/*.cu` is compiled by nvcc with `-gencode arch=compute_100a,
code=sm_100a -lineinfo -O3` into `_build/`, then linked into
`hexlib_b200/_lib/libhexlib_b200.so` against the CUDA runtime (static) alone:
the one driver-API function used, cuTensorMapEncodeTiled, is fetched at run
time through cudaGetDriverEntryPoint. Objects are rebuilt only when a source
or header is newer than them, so calling `build()` on every import is cheap.

The library is built into the package directory (not site-packages, not a JIT
cache) so that it travels with the source tree and is the file a process
loads.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD_DIR = os.path.join(ROOT, "_build", "hexlib_b200")
LIB_DIR = os.path.join(HERE, "_lib")
LIB_NAME = "libhexlib_b200.so"
LIB_PATH = os.path.join(LIB_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
    "-Xcompiler", "-Wall", "-Xcompiler", "-Wno-unused-function",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"),
                 "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin on PATH")


def _sources() -> list[str]:
    return sorted(
        os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu")
    )


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC)
          if f.endswith((".h", ".cuh"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)
           if f.endswith(".h")]
    return hs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(nvcc: str, src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", INCLUDE, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)
    return obj


def build(verbose: bool = False) -> str:
    """Compile every kernel and the C ABI; return the path of the library."""
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    srcs = _sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, verbose), srcs))
    if _stale(LIB_PATH, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", LIB_PATH, *objs,
               "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
