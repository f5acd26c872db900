"""Builds the native libraries of the B200 backend in-tree.

    python -m pyflamert_b200.build          # everything that can be built here

Outputs (git-ignored, shipped with the source tree to the GPU machine):

* ``pyflamert_b200/lib/libpfrt_cuda.so`` -- the C ABI (``include/pfrt_cuda.h``)
  over the sm_100a kernels in ``pyflamert_b200/csrc``.  nvcc cross-compiles
  for ``sm_100a`` without a GPU.  The CUDA runtime is linked statically so the
  library has no dependency beyond the NVIDIA driver.
* ``pyflamert_b200/lib/libpfrt_cuda_backend.so`` -- the PyFlameRT ``Backend``
  implementation (``pyflamert_b200/backend``), compiled against the PyFlameRT
  public headers when they are available (``PYFLAMERT_INCLUDE`` or the default
  reference location).  Its PyFlameRT symbols are resolved by the host
  process that loads it, as with any runtime plugin.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "lib")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _run(cmd, cwd=None):
    r = subprocess.run(cmd, cwd=cwd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}")
    return r.stdout


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_cuda(verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.hpp"))
                     + glob.glob(os.path.join(INCLUDE, "*.h")))
    objs = []
    jobs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if _stale(o, [s] + headers):
            cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else []) + ["-c", s, "-o", o]
            jobs.append(cmd)
    out = []
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for res in ex.map(_run, jobs):
            out.append(res)
    so = os.path.join(LIB, "libpfrt_cuda.so")
    if jobs or _stale(so, objs):
        _run([nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", so] + objs + ["-lpthread", "-ldl", "-lrt"])
    if verbose:
        print("\n".join(x for x in out if x.strip()))
    return so


def reference_include() -> str | None:
    cand = os.environ.get("PYFLAMERT_INCLUDE", "/root/reference/include")
    return cand if os.path.isdir(os.path.join(cand, "pyflame_rt")) else None


def build_backend() -> str | None:
    """The PyFlameRT Backend plugin (needs the PyFlameRT headers)."""
    inc = reference_include()
    srcs = sorted(glob.glob(os.path.join(PKG, "backend", "*.cpp")))
    if inc is None or not srcs:
        return None
    os.makedirs(LIB, exist_ok=True)
    so = os.path.join(LIB, "libpfrt_cuda_backend.so")
    hdrs = glob.glob(os.path.join(PKG, "backend", "*.hpp")) + [os.path.join(INCLUDE, "pfrt_cuda.h")]
    if _stale(so, srcs + hdrs + [os.path.join(LIB, "libpfrt_cuda.so")]):
        cxx = os.environ.get("CXX", "g++")
        _run([cxx, "-std=c++17", "-O2", "-fPIC", "-shared", f"-I{INCLUDE}", f"-I{inc}",
              f"-I{os.path.join(PKG, 'backend')}", "-o", so] + srcs
             + [f"-L{LIB}", "-lpfrt_cuda", "-Wl,-rpath,$ORIGIN"])
    return so


def build_oracle() -> None:
    _run(["make", "-s", "-C", os.path.join(ROOT, "oracle")])


def build_all(verbose: bool = False) -> None:
    build_cuda(verbose=verbose)
    build_backend()
    build_oracle()


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv)
    print("built:", ", ".join(sorted(os.listdir(LIB))))
