"""Build the reference's own CUDA extension, renamed, as a GPU-side checker and
"kernel to beat" -- TEST INFRASTRUCTURE ONLY.

    python oracle/build_ref_cuda.py

Compiles src/cpp/binding.cpp and src/cpp/delta_kernel.cu where they lie in the
reference checkout (the directory in ``DELTAGRID_REF``, ``oracle/refpath.py``) with
torch.utils.cpp_extension for sm_100a, under the module name
``ref_hsru_delta_cuda`` (binding.cpp:523 registers TORCH_EXTENSION_NAME, so the
rename needs no source change).  All outputs go to oracle/_ref/, which is
git-ignored and travels to the GPU box with the tree.  Nothing is copied from
the reference into the repository.
"""
from __future__ import annotations

import glob
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "ref_hsru_delta_cuda"


def build() -> str:
    sys.path.insert(0, HERE)
    from refpath import reference_root
    ref = reference_root()
    src = os.path.join(ref, "src", "cpp")
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    os.environ.setdefault("MAX_JOBS", "8")
    from torch.utils.cpp_extension import load
    bdir = os.path.join(OUT, "cuda_build")
    os.makedirs(bdir, exist_ok=True)
    load(name=NAME, sources=[os.path.join(src, "binding.cpp"), os.path.join(src, "delta_kernel.cu")],
         extra_cflags=["-O3"], extra_cuda_cflags=["-O3", "-gencode=arch=compute_100a,code=sm_100a"],
         build_directory=bdir, verbose=False, with_cuda=True)
    so = glob.glob(os.path.join(bdir, NAME + "*.so"))[0]
    dst = os.path.join(OUT, NAME + ".so")
    shutil.copy2(so, dst)
    return dst


def load_prebuilt():
    """Import the prebuilt module from oracle/_ref (returns None when absent)."""
    import importlib.util
    path = os.path.join(OUT, NAME + ".so")
    if not os.path.exists(path):
        return None
    import torch  # noqa: F401  (the extension links against libtorch)
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build())
    sys.exit(0)
