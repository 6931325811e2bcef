"""In-tree build of the native parts of the B200 long-context attention package.

Produces, next to the Python package (so the built files travel with the tree):

* ``python/long_context_attention/liblca_b200.so`` -- the C ABI of ``include/lca.h``:
  the sm_100a kernels plus the host layer (nvcc, ``-gencode arch=compute_100a,code=sm_100a``,
  static CUDA runtime);
* ``python/long_context_attention_kernels<EXT_SUFFIX>`` -- the torch extension module with
  the reference's name, linked against ``liblca_b200.so`` (rpath ``$ORIGIN/long_context_attention``).

Usage: ``python long-context-attention-kernels_b200/build_native.py [--force]``.
Rebuilds only what is older than its sources unless ``--force`` is given.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
PYDIR = os.path.join(HERE, "python")
PKGDIR = os.path.join(PYDIR, "long_context_attention")
INCLUDE = os.path.join(REPO, "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_HOME = os.path.dirname(os.path.dirname(NVCC))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CABI_SOURCES = ["swa_kernels.cu", "swa_backward.cu", "capi.cpp", "noalloc.cu"]
CABI_HEADERS = ["sm100_ptx.cuh", "swa_kernels.h", "swa_backward.h", "trace.cuh"]
LIB_NAME = "liblca_b200.so"
TRACE_LIB_NAME = "liblca_b200_trace.so"  # -DLCA_TRACE: in-kernel event trace (trace.cuh)
EXT_NAME = "long_context_attention_kernels"


def lib_path() -> str:
    return os.path.join(PKGDIR, LIB_NAME)


def ext_path() -> str:
    return os.path.join(PYDIR, EXT_NAME + sysconfig.get_config_var("EXT_SUFFIX"))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_cabi(force: bool = False, verbose_ptxas: bool = False, trace: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in CABI_SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in CABI_HEADERS] + [os.path.join(INCLUDE, "lca.h")]
    out = os.path.join(PKGDIR, TRACE_LIB_NAME) if trace else lib_path()
    if not force and not _stale(out, deps):
        return out
    tmp = out + ".tmp"
    cmd = [NVCC, "-std=c++17", "-O3", *ARCH, "-lineinfo", "-shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-cudart", "static", f"-I{INCLUDE}", f"-I{CSRC}",
           "-DLCA_BUILDING_LIBRARY", "-o", tmp, *srcs]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    if trace:
        cmd.insert(1, "-DLCA_TRACE")
    _run(cmd)
    os.replace(tmp, out)
    return out


def build_extension(force: bool = False) -> str:
    import torch.utils.cpp_extension as ce
    import torch

    src = os.path.join(CSRC, "bindings.cpp")
    deps = [src, os.path.join(INCLUDE, "lca.h"), lib_path()]
    out = ext_path()
    if not force and not _stale(out, deps):
        return out
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [f"-I{p}" for p in ce.include_paths()] + [f"-I{sysconfig.get_paths()['include']}",
                                                      f"-I{CUDA_HOME}/include", f"-I{INCLUDE}"]
    libs = [f"-L{p}" for p in ce.library_paths()] + [f"-L{PKGDIR}"]
    tmp = out + ".tmp"
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={EXT_NAME}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", *incs, src, "-o", tmp, *libs,
           "-l:" + LIB_NAME, "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
           "-Wl,-rpath,$ORIGIN/long_context_attention"]
    _run(cmd)
    os.replace(tmp, out)
    return out


def build(force: bool = False, verbose_ptxas: bool = False) -> None:
    build_cabi(force=force, verbose_ptxas=verbose_ptxas)
    build_extension(force=force)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    ap.add_argument("--trace", action="store_true",
                    help=f"also build {TRACE_LIB_NAME}, the C ABI with the in-kernel event trace")
    a = ap.parse_args(argv)
    build(force=a.force, verbose_ptxas=a.ptxas_verbose)
    if a.trace:
        build_cabi(force=a.force, verbose_ptxas=a.ptxas_verbose, trace=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
