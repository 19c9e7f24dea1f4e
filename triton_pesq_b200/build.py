"""In-tree build of the CUDA engine for sm_100a.

Produces, next to this file:

* ``libpesq_cuda.so`` -- the kernels and the C ABI of ``include/pesq_cuda.h``
  (nvcc, ``-gencode arch=compute_100a,code=sm_100a``, static cudart);
* ``_pesq_torch_ops.so`` -- the ``torch.ops.pesq_cuda`` custom ops, a thin
  layer over the C ABI (built with ``torch.utils.cpp_extension``).

Usage: ``python -m triton_pesq_b200.build`` (or ``__graft_entry__.build()``).
nvcc cross-compiles without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libpesq_cuda.so")
OPS = os.path.join(HERE, "_pesq_torch_ops.so")

CUDA_SOURCES = ["front.cu", "align.cu", "back.cu", "spectrum.cu", "chain.cu", "resample.cu", "pesq_abi.cu", "noalloc.cu",
                "resample_abi.cu", "iir_abi.cu", "iir_ka.cu", "iir_kb.cu", "iir_kc.cu", "iir_kd.cu", "iir_ke.cu",
                "iir_kf.cu"]
NVCC_FLAGS = [
    "-std=c++17",
    "-O3",
    "-lineinfo",
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-v",
    f"-I{os.path.join(ROOT, 'include')}",
]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(home, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def _run(cmd, log):
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    with open(log, "w") as fh:
        fh.write(" ".join(cmd) + "\n" + proc.stdout)
    if proc.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{proc.stdout}")
    return proc.stdout


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _deps():
    out = [os.path.join(ROOT, "include", "pesq_cuda.h")]
    for name in os.listdir(CSRC):
        if name.endswith((".cu", ".cuh", ".cpp", ".h")):
            out.append(os.path.join(CSRC, name))
    return out


def build_library(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    deps = _deps()
    if not force and not _stale(LIB, deps):
        return LIB
    nvcc = _nvcc()

    def compile_one(src):
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        out = _run([nvcc, *NVCC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj],
                   os.path.join(BUILD, src + ".log"))
        if verbose:
            print(out)
        return obj

    with ThreadPoolExecutor(max_workers=len(CUDA_SOURCES)) as pool:
        objs = list(pool.map(compile_one, CUDA_SOURCES))
    tmp = LIB + ".tmp"
    _run([nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-Xlinker", "-soname=libpesq_cuda.so",
          *objs, "-o", tmp],
         os.path.join(BUILD, "link.log"))
    os.replace(tmp, LIB)
    return LIB


def build_torch_ops(force: bool = False, verbose: bool = False) -> str:
    deps = _deps() + [LIB]
    if not force and not _stale(OPS, deps):
        return OPS
    from torch.utils import cpp_extension

    bdir = os.path.join(BUILD, "torch_ops")
    os.makedirs(bdir, exist_ok=True)
    # load() imports the result from the build directory, where $ORIGIN does
    # not reach libpesq_cuda.so: make it resolvable by soname first
    import ctypes

    ctypes.CDLL(LIB, mode=ctypes.RTLD_GLOBAL)
    cpp_extension.load(
        name="pesq_torch_ops",
        sources=[os.path.join(CSRC, "torch_ops.cpp")],
        extra_cflags=["-O2", "-std=c++17"],
        extra_ldflags=[f"-L{HERE}", "-lpesq_cuda", "-Wl,-rpath,\\$$ORIGIN"],
        build_directory=bdir,
        with_cuda=True,
        is_python_module=False,
        verbose=verbose,
    )
    shutil.copyfile(os.path.join(bdir, "pesq_torch_ops.so"), OPS + ".tmp")
    os.replace(OPS + ".tmp", OPS)
    return OPS


def build(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    if force or _stale(OPS, _deps() + [LIB]):
        # cpp_extension.load() registers the ops from its build directory:
        # compile in a child process so that this one can still load the
        # in-tree copy (a namespace may be registered only once per process)
        code = f"from triton_pesq_b200.build import build_torch_ops; build_torch_ops(force=True, verbose={verbose!r})"
        subprocess.run([sys.executable, "-c", code], check=True, cwd=os.path.dirname(HERE))


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
    print(OPS)
