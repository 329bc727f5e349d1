"""Build recipe for the reference GEMV kernel, compiled from its own source file.

TEST INFRASTRUCTURE ONLY.  The product never loads what this builds.

The reference (Naturalseeker22/Nvidia-x-GPU-MODE-Kernels) is a single PyTorch
C++/CUDA extension, ``blackwell_nvfp4_gemv.cu``, exporting
``nvfp4_gemv_forward(a, b, sa, sb, c, M, K, L)`` through pybind
(``blackwell_nvfp4_gemv.cu:500-524``).  It ships no build script, so this file
is the build line: nvcc for sm_100a on the source where it lies, then a
g++ link against libtorch.  The output goes to ``oracle/_ref/`` (git-ignored,
but it travels to the GPU box with the rest of the tree).

The built module is used in two places only:

* the ``-m gpu`` tests, to pin the CPU oracle against the reference kernel's own
  outputs and to compare the new kernels with it on the same inputs;
* ``tests/golden/make_golden.py``, which records the reference kernel's outputs
  as committed fixtures so the CPU-only tests can pin the oracle too.

Nothing here reads the reference at run time on the GPU box: the ``.so`` is
built in the development container, where the source exists.  The source file
is named by ``--src PATH`` or the ``NVFP4_REF_SRC`` environment variable; with
neither, an already built module is kept and nothing is compiled.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
REF_SRC = os.environ.get("NVFP4_REF_SRC")
MODULE = "ref_nvfp4_gemv"
SO_PATH = os.path.join(OUT_DIR, MODULE + sysconfig.get_config_var("EXT_SUFFIX"))


def _torch_paths():
    import torch
    tdir = os.path.dirname(torch.__file__)
    inc = [os.path.join(tdir, "include"),
           os.path.join(tdir, "include", "torch", "csrc", "api", "include")]
    return inc, os.path.join(tdir, "lib"), torch.compiled_with_cxx11_abi()


def build(force: bool = False, verbose: bool = False, src: str | None = None) -> str | None:
    """Compile the reference source ``src`` (default: ``NVFP4_REF_SRC``) into
    ``oracle/_ref``.  Returns the .so path, or None when no source is named or
    it is absent (as on the GPU box) and nothing was built before."""
    src = src or REF_SRC
    if not src or not os.path.exists(src):
        return SO_PATH if os.path.exists(SO_PATH) else None
    if (not force and os.path.exists(SO_PATH)
            and os.path.getmtime(SO_PATH) >= os.path.getmtime(src)
            and os.path.getmtime(SO_PATH) >= os.path.getmtime(__file__)):
        return SO_PATH
    os.makedirs(OUT_DIR, exist_ok=True)
    inc, libdir, cxx11 = _torch_paths()
    py_inc = sysconfig.get_paths()["include"]
    obj = os.path.join(OUT_DIR, MODULE + ".o")
    defs = [f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H",
            f"-D_GLIBCXX_USE_CXX11_ABI={int(cxx11)}"]
    nvcc = ["nvcc", "-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a",
            "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", *defs,
            *[f"-I{p}" for p in inc], f"-I{py_inc}", "-c", src, "-o", obj]
    link = ["g++", "-shared", "-o", SO_PATH, obj, f"-L{libdir}", "-lc10", "-lc10_cuda",
            "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
            "-L/usr/local/cuda/lib64", "-lcudart", f"-Wl,-rpath,{libdir}"]
    for cmd in (nvcc, link):
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    os.remove(obj)
    return SO_PATH


def load():
    """Import the built reference module (needs torch imported first)."""
    import importlib.machinery
    import importlib.util
    import torch  # noqa: F401  (libtorch must be loaded before the extension)
    if not os.path.exists(SO_PATH):
        raise FileNotFoundError(f"reference GEMV not built: {SO_PATH}")
    loader = importlib.machinery.ExtensionFileLoader(MODULE, SO_PATH)
    spec = importlib.util.spec_from_file_location(MODULE, SO_PATH, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    args = sys.argv[1:]
    src = args[args.index("--src") + 1] if "--src" in args else None
    p = build(force="--force" in args, verbose=True, src=src)
    print(p)
