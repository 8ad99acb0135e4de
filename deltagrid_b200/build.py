"""Builds the native parts in-tree.

    python -m deltagrid_b200.build          (or deltagrid_b200.build.build())

1. libdeltagrid_b200.so: every .cu under csrc/ compiled with nvcc for sm_100a in
   parallel, and the host-only .cpp sources (all but binding.cpp) through nvcc's
   host compiler, then linked into a shared library next to this file (the C ABI
   of include/deltagrid_b200.h).
2. _hsru<ext suffix>: csrc/binding.cpp, the compiled torch extension behind
   deltagrid_b200.hsru_delta_cuda, built with the host C++ compiler against
   torch's headers and linked to libdeltagrid_b200.so (found next to it at run time).

Rebuilds only what changed (by mtime, including the shared headers).
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libdeltagrid_b200.so")
BINDING_SRC = os.path.join(CSRC, "binding.cpp")
BINDING = os.path.join(HERE, "_hsru" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                     "-Xptxas", "-warn-spills", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _headers_mtime() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OBJ, os.path.splitext(os.path.basename(src))[0] + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), _headers_mtime()):
        return obj
    cmd = [nvcc()] + NVCC_FLAGS + ["-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, file=sys.stderr)
    return obj


def _build_binding() -> str:
    """The torch extension module `_hsru` (needs torch's headers and libraries, no GPU)."""
    deps = [BINDING_SRC, LIB, os.path.join(INCLUDE, "deltagrid_b200.h")]
    if os.path.exists(BINDING) and os.path.getmtime(BINDING) >= max(os.path.getmtime(d) for d in deps):
        return BINDING
    import torch
    tdir = os.path.dirname(torch.__file__)
    tinc = os.path.join(tdir, "include")
    tlib = os.path.join(tdir, "lib")
    cuda_home = os.path.dirname(os.path.dirname(os.path.realpath(nvcc())))
    cxx = os.environ.get("CXX") or shutil.which("g++") or "c++"
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", BINDING_SRC, "-o", BINDING,
           f"-I{tinc}", f"-I{os.path.join(tinc, 'torch', 'csrc', 'api', 'include')}",
           f"-I{os.path.join(cuda_home, 'include')}", f"-I{sysconfig.get_paths()['include']}", f"-I{INCLUDE}",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}", "-DTORCH_EXTENSION_NAME=_hsru",
           "-DTORCH_API_INCLUDE_EXTENSION_H", f"-L{tlib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_python", f"-L{HERE}", "-ldeltagrid_b200", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{tlib}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"binding build failed:\n{r.stdout}\n{r.stderr}")
    return BINDING


def build(verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    srcs += sorted(p for p in glob.glob(os.path.join(CSRC, "*.cpp")) if p != BINDING_SRC)
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart", "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    _build_binding()
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
