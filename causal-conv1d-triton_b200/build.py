"""Builds libcausal_conv1d_b200.so (the C-ABI library of include/causal_conv1d_b200.h) for
sm_100a with nvcc, in-tree: objects under _build/, the library inside the Python package; then the
package's CPython binding of the hot entry points (csrc/cc1d_pyfast.c -> _cc1d_fast*.so) and its
torch-side forward/backward launchers (csrc/cc1d_torch_ext.cpp -> _cc1d_torch*.so, host C++ against
torch's headers), both linked against that library.

    python causal-conv1d-triton_b200/build.py [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "causal_conv1d_b200", "libcausal_conv1d_b200.so")
FAST_SRC = os.path.join(CSRC, "cc1d_pyfast.c")
FAST = os.path.join(HERE, "causal_conv1d_b200", "_cc1d_fast" + sysconfig.get_config_var("EXT_SUFFIX"))
TORCH_SRC = os.path.join(CSRC, "cc1d_torch_ext.cpp")
TORCH_EXT = os.path.join(HERE, "causal_conv1d_b200", "_cc1d_torch" + sysconfig.get_config_var("EXT_SUFFIX"))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
    "-I", INCLUDE, "-I", CSRC,
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build")
    return cand


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]


def _stale(target, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False,
          defines: tuple = (), lib_path: str = LIB, build_dir: str = BUILD) -> str:
    """Compiles every .cu under csrc/ for sm_100a and links the shared library; returns its path.

    `defines` (e.g. ("CC1D_BWD_LAG=1",)) override the kernels' compile-time tuning constants; use
    them with a separate `lib_path` and `build_dir`."""
    os.makedirs(build_dir, exist_ok=True)
    nvcc = _nvcc()
    headers = _headers()
    srcs = sources()
    objs = [os.path.join(build_dir, os.path.basename(s)[:-3] + ".o") for s in srcs]
    dflags = [f"-D{d}" for d in defines]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or ptxas_verbose or _stale(o, [s] + headers)]

    def compile_one(so):
        s, o = so
        cmd = [nvcc] + NVCC_FLAGS + dflags + (["-Xptxas", "-v"] if ptxas_verbose else []) + ["-c", s, "-o", o]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {s}:\n{r.stdout}\n{r.stderr}")
        return s, r.stderr

    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            for s, err in ex.map(compile_one, todo):
                if ptxas_verbose and err:
                    print(f"== {os.path.basename(s)}\n{err}", flush=True)
    if force or todo or _stale(lib_path, objs):
        cmd = [nvcc] + ARCH + ["-shared", "-Xlinker", "-soname=libcausal_conv1d_b200.so", "-o", lib_path] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if lib_path == LIB:
        build_fast(force, verbose)
        build_torch_ext(force, verbose)
    return lib_path


def build_fast(force: bool = False, verbose: bool = False) -> str:
    """Compiles the CPython binding (C, no CUDA code) against the built library."""
    header = os.path.join(INCLUDE, "causal_conv1d_b200.h")
    if not (force or _stale(FAST, [FAST_SRC, header, LIB])):
        return FAST
    cc = shutil.which("gcc") or "cc"
    cmd = [cc, "-O2", "-fPIC", "-shared", "-std=c11", "-Wall", "-Wextra",
           "-I", sysconfig.get_paths()["include"], "-I", INCLUDE, FAST_SRC,
           "-L", os.path.dirname(LIB), "-lcausal_conv1d_b200", "-Wl,-rpath,$ORIGIN", "-o", FAST]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"binding build failed:\n{r.stdout}\n{r.stderr}")
    return FAST


def build_torch_ext(force: bool = False, verbose: bool = False) -> str:
    """Compiles the torch-side launchers (host C++, torch's headers and libraries) against the built
    library."""
    header = os.path.join(INCLUDE, "causal_conv1d_b200.h")
    if not (force or _stale(TORCH_EXT, [TORCH_SRC, header, LIB])):
        return TORCH_EXT
    import torch
    import torch.utils.cpp_extension as ce

    cxx = shutil.which("g++") or "c++"
    torch_lib = ce.library_paths()[0]
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(_nvcc())), "include")
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch.compiled_with_cxx11_abi())}",
           "-DTORCH_EXTENSION_NAME=_cc1d_torch", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    for inc in ce.include_paths() + [cuda_inc, sysconfig.get_paths()["include"], INCLUDE]:
        cmd += ["-I", inc]
    cmd += [TORCH_SRC, "-L", os.path.dirname(LIB), "-lcausal_conv1d_b200", "-L", torch_lib, "-lc10", "-lc10_cuda",
            "-ltorch", "-ltorch_cpu", "-ltorch_python", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}",
            "-o", TORCH_EXT]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch launcher build failed:\n{r.stdout}\n{r.stderr}")
    return TORCH_EXT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas_verbose))
    sys.exit(0)
