"""Build libtfattn.so (the C-ABI library of the hot path) in-tree with nvcc for sm_100a.

    python -m tokenfactory_b200.build [--verbose-ptxas] [--jobs N]

Every csrc/*.cu is compiled to an object under tokenfactory_b200/_build/ (in parallel, only when the
source or a header is newer than the object), then linked with the static CUDA runtime into
tokenfactory_b200/libtfattn.so.  A linker version script exports only the tf_* symbols declared in
include/tfattn.h, so the library's private copy of the runtime never clashes with torch's.  Then
csrc/torch_ext.cpp, the PyTorch front end over that C ABI, is compiled into
tokenfactory_b200/_C.<python ext suffix>.so.
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


def _ext_path() -> str:
    import sysconfig
    return os.path.join(PKG, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_torch_ext() -> str:
    """The PyTorch front end (tokenfactory_b200._C, csrc/torch_ext.cpp): a host C++ module over
    libtfattn.so's C ABI, compiled with the host compiler against torch's headers and libraries,
    linked to libtfattn.so through an $ORIGIN run path.  Returns the module's path."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension as ce

    src = os.path.join(CSRC, "torch_ext.cpp")
    out = _ext_path()
    newest = max(os.path.getmtime(src), os.path.getmtime(LIB), _headers_mtime())
    if os.path.exists(out) and os.path.getmtime(out) >= newest:
        return out
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-I", INCLUDE,
           "-I", sysconfig.get_paths()["include"]]
    for inc in ce.include_paths(device_type="cuda"):
        cmd += ["-isystem", inc]
    cmd += [src, "-o", out + ".tmp"]
    for lib_dir in ce.library_paths(device_type="cuda"):
        cmd += ["-L", lib_dir]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
            "-L", PKG, "-l:libtfattn.so", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch extension build failed:\n{r.stderr[-4000:]}")
    os.replace(out + ".tmp", out)
    return out


def build(verbose_ptxas: bool = False, jobs: int = 0) -> str:
    """Compile and link libtfattn.so, then the torch front end over it; returns the library path."""
    lib = build_lib(verbose_ptxas, jobs)
    build_torch_ext()
    return lib


def build_lib(verbose_ptxas: bool = False, jobs: int = 0) -> str:
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
