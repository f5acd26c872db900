"""Builds the native libraries of the B200 backend in-tree.

    python -m pyflamert_b200.build          # everything that can be built here

Outputs (git-ignored, shipped with the source tree to the GPU machine):

* ``pyflamert_b200/lib/libpfrt_cuda.so`` -- the C ABI (``include/pfrt_cuda.h``)
  over the sm_100a kernels in ``pyflamert_b200/csrc``.  nvcc cross-compiles
  for ``sm_100a`` without a GPU.  The CUDA runtime is linked statically so the
  library has no dependency beyond the NVIDIA driver.
* ``pyflamert_b200/lib/libpfrt_cuda_backend.so`` -- the PyFlameRT ``Backend``
  implementation (``pyflamert_b200/backend``), compiled against the PyFlameRT
  public headers when they are available (``PYFLAMERT_INCLUDE``, by default a
  PyFlameRT checkout named ``reference`` beside this repository).  Its
  PyFlameRT symbols are resolved by the host process that loads it, as with
  any runtime plugin.
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


def cxx() -> str:
    """The C++ compiler for the host-side libraries: PFRT_CXX, else the g++ on
    PATH.  The CXX variable is not used: these libraries are loaded into
    processes that already hold the system's shared libstdc++ (Python, the
    PyFlameRT runtime), so they must link it too; a toolchain that links
    libstdc++ statically gives each library its own copy of the iostream and
    locale internals, and streams then break across the library boundary."""
    return os.environ.get("PFRT_CXX") or shutil.which("g++") or "g++"


def cc() -> str:
    return os.environ.get("PFRT_CC") or shutil.which("gcc") or "gcc"


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
    """PyFlameRT's public headers: PYFLAMERT_INCLUDE, by default the include/
    directory of a checkout named "reference" beside this repository."""
    cand = os.environ.get("PYFLAMERT_INCLUDE", os.path.join(os.path.dirname(ROOT), "reference", "include"))
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
        compiler = cxx()
        _run([compiler, "-std=c++17", "-O2", "-fPIC", "-shared", f"-I{INCLUDE}", f"-I{inc}",
              f"-I{os.path.join(PKG, 'backend')}", "-o", so] + srcs
             + [f"-L{LIB}", "-lpfrt_cuda", "-Wl,-rpath,$ORIGIN"])
    return so


def build_oracle() -> None:
    _run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"CXX={cxx()}", f"CC={cc()}"])


def build_native_tests() -> str | None:
    """tests/native/test_cuda_backend: the Backend plugin against the
    reference's CPUExecutor (test infrastructure; needs the reference headers
    and oracle/_ref)."""
    inc = reference_include()
    ref_lib = os.path.join(ROOT, "oracle", "_ref", "libpfrt_ref.so")
    src = os.path.join(ROOT, "tests", "native", "test_cuda_backend.cpp")
    if inc is None or not os.path.exists(ref_lib) or not os.path.exists(src):
        return None
    out_dir = os.path.join(ROOT, "tests", "native", "_build")
    os.makedirs(out_dir, exist_ok=True)
    exe = os.path.join(out_dir, "test_cuda_backend")
    deps = [src, ref_lib, os.path.join(LIB, "libpfrt_cuda_backend.so")]
    if _stale(exe, deps):
        compiler = cxx()
        ref_src = os.path.join(os.path.dirname(inc), "src")
        _run([compiler, "-std=c++17", "-O2", f"-I{inc}", f"-I{ref_src}", f"-I{INCLUDE}",
              f"-I{os.path.join(PKG, 'backend')}", f"-I{os.path.join(ROOT, 'oracle')}", "-o", exe, src,
              f"-L{LIB}", "-lpfrt_cuda_backend", "-lpfrt_cuda",
              f"-L{os.path.dirname(ref_lib)}", "-lpfrt_ref",
              f"-L{os.path.join(ROOT, 'oracle', '_build')}", "-loracle",
              "-Wl,-rpath,$ORIGIN/../../../pyflamert_b200/lib:$ORIGIN/../../../oracle/_ref:"
              "$ORIGIN/../../../oracle/_build",
              "-lpthread"])
    return exe


# The session seam: the edits that let SessionOptions.device = "cuda" or
# "cuda:<n>[,<m>...]" select the CudaBackend (src/options.cpp:12-17,
# src/session.cpp:67-95).  "cuda" takes its devices from PFRT_CUDA_DEVICES
# (default device 0); make_cuda_backend(device string) parses them.
SEAM_EDITS = {
    "src/options.cpp": [
        ('"cpu", "wse", "wse2", "wse3"', '"cpu", "cuda", "wse", "wse2", "wse3"'),
        ("if (valid_devices.find(device) == valid_devices.end()) {",
         "if (valid_devices.find(device) == valid_devices.end() && device.rfind(\"cuda:\", 0) != 0) {"),
    ],
    "src/session.cpp": [
        ('if (options_.device != "cpu") {', 'if (options_.device != "cpu" && options_.device.rfind("cuda", 0) != 0) {'),
        ("    backend_ = std::make_unique<CPUExecutor>(",
         "    if (options_.device.rfind(\"cuda\", 0) == 0) {\n"
         "        backend_ = ::pyflame_rt::make_cuda_backend(options_.device);\n"
         "        return;\n"
         "    }\n"
         "    backend_ = std::make_unique<CPUExecutor>("),
    ],
}

SESSION_SRCS = ["src/io/loader.cpp", "src/io/pyflame_format.cpp", "src/quantization/calibrator.cpp",
                "src/opt/pass_manager.cpp", "src/opt/layout_optimization.cpp"]


def build_session_test() -> str | None:
    """tests/native/test_session_seam: the reference's InferenceSession, with
    the seam edits applied to copies of its sources, running device="cuda"
    against device="cpu".  Test infrastructure; needs the reference sources."""
    inc = reference_include()
    ref_lib = os.path.join(ROOT, "oracle", "_ref", "libpfrt_ref.so")
    src = os.path.join(ROOT, "tests", "native", "test_session_seam.cpp")
    if inc is None or not os.path.exists(ref_lib) or not os.path.exists(src):
        return None
    ref = os.path.dirname(inc)
    out_dir = os.path.join(ROOT, "tests", "native", "_build")
    os.makedirs(out_dir, exist_ok=True)
    exe = os.path.join(out_dir, "test_session_seam")
    stubs = os.path.join(PKG, "session", "pass_stubs.cpp")
    deps = [src, stubs, ref_lib, os.path.join(LIB, "libpfrt_cuda_backend.so")]
    if not _stale(exe, deps):
        return exe
    import tempfile
    srcs = [src, stubs] + [os.path.join(ref, f) for f in SESSION_SRCS]
    with tempfile.TemporaryDirectory() as tmp:  # patched copies never enter the tree
        srcs += _patched_seam_sources(ref, tmp)
        compiler = cxx()
        _run([compiler, "-std=c++17", "-O2", "-w", f"-I{inc}", f"-I{os.path.join(ref, 'src')}", f"-I{INCLUDE}",
              f"-I{os.path.join(PKG, 'backend')}", "-include", "pyflame_rt/tensor.hpp", "-include",
              "cuda_backend.hpp", "-o", exe] + srcs +
             [f"-L{LIB}", "-lpfrt_cuda_backend", "-lpfrt_cuda", f"-L{os.path.dirname(ref_lib)}", "-lpfrt_ref",
              "-Wl,-rpath,$ORIGIN/../../../pyflamert_b200/lib:$ORIGIN/../../../oracle/_ref", "-lpthread"])
    return exe


def _patched_seam_sources(ref: str, tmp: str) -> list:
    """Copies of the reference's options.cpp and session.cpp with SEAM_EDITS
    applied, written under `tmp` (the reference tree is never written)."""
    out = []
    for rel, edits in SEAM_EDITS.items():
        text = open(os.path.join(ref, rel)).read()
        for old, new in edits:
            if old not in text:
                raise RuntimeError(f"seam edit does not apply to {rel}: {old!r}")
            text = text.replace(old, new, 1)
        patched = os.path.join(tmp, os.path.basename(rel))
        with open(patched, "w") as f:
            f.write(text)
        out.append(patched)
    return out


# The reference's runtime translation units the session layer needs (the CPU
# operator sources register the CPU backend's ops; the session can still be
# opened on device "cpu").
RUNTIME_SRCS = [
    "src/tensor.cpp", "src/node.cpp", "src/graph.cpp", "src/registry.cpp", "src/backends/cpu/executor.cpp",
    "src/backends/cpu/ops/math.cpp", "src/backends/cpu/ops/activation.cpp", "src/backends/cpu/ops/tensor_ops.cpp",
    "src/backends/cpu/ops/reduction.cpp", "src/backends/cpu/ops/nn.cpp", "src/backends/cpu/ops/quantized_ops.cpp",
    "src/quantization/quant_ops.cpp", "src/quantization/quant_params.cpp", "src/quantization/half_types.cpp",
]


def build_session_lib() -> str | None:
    """pyflamert_b200/lib/libpfrt_session.so: PyFlameRT's InferenceSession
    (its own sources, from the checkout PYFLAMERT_INCLUDE points into) with
    the CUDA seam, and the C entry points of include/pfrt_session.h.  This is
    the host a C/ctypes caller runs the drop-in through; it is built only when
    the PyFlameRT sources are present."""
    inc = reference_include()
    if inc is None:
        return None
    ref = os.path.dirname(inc)
    so = os.path.join(LIB, "libpfrt_session.so")
    own = [os.path.join(PKG, "session", "session_capi.cpp"), os.path.join(PKG, "session", "pass_stubs.cpp")]
    deps = own + [os.path.join(INCLUDE, "pfrt_session.h"), os.path.join(LIB, "libpfrt_cuda_backend.so")]
    if not _stale(so, deps):
        return so
    import tempfile
    srcs = own + [os.path.join(ref, f) for f in RUNTIME_SRCS + SESSION_SRCS]
    with tempfile.TemporaryDirectory() as tmp:
        srcs += _patched_seam_sources(ref, tmp)
        compiler = cxx()
        _run([compiler, "-std=c++17", "-O2", "-w", "-fPIC", "-shared", f"-I{inc}", f"-I{os.path.join(ref, 'src')}",
              f"-I{INCLUDE}", f"-I{os.path.join(PKG, 'backend')}", "-include", "pyflame_rt/tensor.hpp",
              "-include", "cuda_backend.hpp", "-o", so] + srcs +
             [f"-L{LIB}", "-lpfrt_cuda_backend", "-lpfrt_cuda", "-Wl,-rpath,$ORIGIN", "-lpthread"])
    return so


def build_pfm_test() -> str | None:
    """tests/native/test_pfm_fast: PfmImage and CudaBackend::prepare against
    the reference's PyFlameFormat (src/io/pyflame_format.cpp, compiled from the
    reference's sources into the test).  Test infrastructure."""
    inc = reference_include()
    ref_lib = os.path.join(ROOT, "oracle", "_ref", "libpfrt_ref.so")
    src = os.path.join(ROOT, "tests", "native", "test_pfm_fast.cpp")
    if inc is None or not os.path.exists(ref_lib) or not os.path.exists(src):
        return None
    ref = os.path.dirname(inc)
    out_dir = os.path.join(ROOT, "tests", "native", "_build")
    os.makedirs(out_dir, exist_ok=True)
    exe = os.path.join(out_dir, "test_pfm_fast")
    deps = [src, ref_lib, os.path.join(LIB, "libpfrt_cuda_backend.so")]
    if _stale(exe, deps):
        compiler = cxx()
        _run([compiler, "-std=c++17", "-O2", "-w", f"-I{inc}", f"-I{os.path.join(ref, 'src')}", f"-I{INCLUDE}",
              f"-I{os.path.join(PKG, 'backend')}", "-o", exe, src, os.path.join(ref, "src/io/pyflame_format.cpp"),
              f"-L{LIB}", "-lpfrt_cuda_backend", "-lpfrt_cuda", f"-L{os.path.dirname(ref_lib)}", "-lpfrt_ref",
              "-Wl,-rpath,$ORIGIN/../../../pyflamert_b200/lib:$ORIGIN/../../../oracle/_ref", "-lpthread"])
    return exe


def build_batcher_test() -> str | None:
    """tests/native/test_batcher: cuda::DynamicBatcher against each request run
    alone, on the reference's CPUExecutor (CPU) and on CudaBackend (GPU).
    Test infrastructure."""
    inc = reference_include()
    ref_lib = os.path.join(ROOT, "oracle", "_ref", "libpfrt_ref.so")
    src = os.path.join(ROOT, "tests", "native", "test_batcher.cpp")
    if inc is None or not os.path.exists(ref_lib) or not os.path.exists(src):
        return None
    out_dir = os.path.join(ROOT, "tests", "native", "_build")
    os.makedirs(out_dir, exist_ok=True)
    exe = os.path.join(out_dir, "test_batcher")
    deps = [src, ref_lib, os.path.join(LIB, "libpfrt_cuda_backend.so")]
    if _stale(exe, deps):
        compiler = cxx()
        _run([compiler, "-std=c++17", "-O2", "-w", f"-I{inc}", f"-I{os.path.join(os.path.dirname(inc), 'src')}",
              f"-I{INCLUDE}", f"-I{os.path.join(PKG, 'backend')}", "-o", exe, src,
              f"-L{LIB}", "-lpfrt_cuda_backend", "-lpfrt_cuda", f"-L{os.path.dirname(ref_lib)}", "-lpfrt_ref",
              "-Wl,-rpath,$ORIGIN/../../../pyflamert_b200/lib:$ORIGIN/../../../oracle/_ref", "-lpthread"])
    return exe


def build_all(verbose: bool = False) -> None:
    build_cuda(verbose=verbose)
    build_backend()
    build_session_lib()
    build_oracle()
    build_native_tests()
    build_session_test()
    build_pfm_test()
    build_batcher_test()


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv)
    print("built:", ", ".join(sorted(os.listdir(LIB))))
