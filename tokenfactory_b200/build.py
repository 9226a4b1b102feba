"""Build libtfattn.so (the C-ABI library of the hot path) in-tree with nvcc for sm_100a.

    python -m tokenfactory_b200.build [--verbose-ptxas] [--jobs N]

Every csrc/*.cu is compiled to an object under tokenfactory_b200/_build/ (in parallel, only when the
source or a header is newer than the object), then linked with the static CUDA runtime into
tokenfactory_b200/libtfattn.so.  A linker version script exports only the tf_* symbols declared in
include/tfattn.h, so the library's private copy of the runtime never clashes with torch's.
"""

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libtfattn.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler",
              "-fvisibility=hidden", "-I", INCLUDE, "-I", CSRC] + ARCH


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the hot path has no CPU fallback and must be compiled")


def _headers_mtime() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(nvcc: str, src: str, verbose_ptxas: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    newest = max(os.path.getmtime(src), _headers_mtime())
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj
    cmd = [nvcc] + NVCC_FLAGS + ["-c", src, "-o", obj]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stderr}")
    if verbose_ptxas:
        with open(obj + ".ptxas.txt", "w") as f:
            f.write(r.stderr)
    return obj


def build(verbose_ptxas: bool = False, jobs: int = 0) -> str:
    """Compile and link; returns the path of libtfattn.so."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, verbose_ptxas), srcs))
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    vs = os.path.join(BUILD, "exports.map")
    with open(vs, "w") as f:
        f.write("{ global: tf_*; local: *; };\n")
    tmp = LIB + ".tmp"
    cmd = [nvcc, "-shared", "-cudart", "static"] + ARCH + objs + \
        ["-Xlinker", f"--version-script={vs}", "-o", tmp]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--verbose-ptxas", action="store_true",
                    help="record ptxas register/spill/smem reports next to the objects")
    ap.add_argument("--jobs", type=int, default=0)
    args = ap.parse_args()
    print(build(args.verbose_ptxas, args.jobs))


if __name__ == "__main__":
    sys.exit(main())
