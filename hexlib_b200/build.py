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


def _compile(nvcc: str, src: str, verbose: bool, build_dir: str = BUILD_DIR,
             defines: tuple[str, ...] = ()) -> str:
    obj = os.path.join(build_dir, os.path.basename(src)[:-3] + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *(f"-D{d}" for d in defines), "-I", INCLUDE,
           "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)
    return obj


def build(verbose: bool = False, measure: bool = False) -> str:
    """Compile every kernel and the C ABI; return the path of the library.

    `measure` builds the measurement variant instead, into
    _lib/libhexlib_b200_measure.so: the same code with
    HEXLIB_B200_MEASUREMENT_KNOBS defined, so that a few environment
    variables (HEXLIB_B200_GEMM_TILE, HEXLIB_B200_GEMM_PAIR[_RES],
    HEXLIB_B200_WALK_ORDER) can pin a kernel variant for
    an A/B comparison. The shipped library reads no environment."""
    nvcc = _nvcc()
    build_dir = os.path.join(BUILD_DIR, "measure") if measure else BUILD_DIR
    lib_path = os.path.join(LIB_DIR, "libhexlib_b200_measure.so") if measure else LIB_PATH
    defines = ("HEXLIB_B200_MEASUREMENT_KNOBS",) if measure else ()
    os.makedirs(build_dir, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    srcs = _sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, verbose, build_dir, defines), srcs))
    if _stale(lib_path, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", lib_path, *objs,
               "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib_path


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, measure="--measure" in sys.argv))
