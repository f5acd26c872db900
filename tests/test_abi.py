"""The C ABI library without a GPU: it loads, it exports every function that
include/*.h declares, the ctypes prototypes cover them, it fails loudly when
no device is present, and its host-side CSR validation rejects what
SparseTensor::from_csr (src/pruning/sparse_tensor.cpp:170-197) lets through."""
import ctypes as C
import glob
import os
import re
import subprocess

import numpy as np
import pytest

import pyflamert_b200 as pf
from pyflamert_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        names |= set(re.findall(r"^PFRT_API\s+[\w\s\*]+?\b(pfrt_\w+)\s*\(", txt, flags=re.M))
    return names


def test_header_declares_api():
    names = declared_functions()
    assert {"pfrt_ctx_create", "pfrt_qlinear", "pfrt_gemm_f32", "pfrt_spmm"} <= names


def test_library_exports_every_declared_symbol():
    path = pf.lib_path()
    assert os.path.exists(path), "libpfrt_cuda.so must be built (python -m pyflamert_b200.build)"
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(pfrt_\w+)", out))
    missing = declared_functions() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_ctypes_prototypes_cover_header():
    assert declared_functions() == set(_abi.PROTOTYPES)


def test_library_loads_and_reports_version():
    assert b"sm_100a" in pf.lib().pfrt_version()


def test_no_device_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    st = pf.lib().pfrt_ctx_create(0, C.byref(h))
    assert st == 7  # PFRT_ERR_NO_DEVICE
    assert "device" in _abi.last_error().lower()
    with pytest.raises(pf.PfrtError):
        pf.Context(0)


def _validate(N, K, indptr, indices, bits=32):
    dt = np.int32 if bits == 32 else np.int64
    ip = np.ascontiguousarray(indptr, dt)
    ix = np.ascontiguousarray(indices, dt)
    return pf.lib().pfrt_csr_validate_host(N, K, ix.size, ip.ctypes.data_as(C.c_void_p),
                                           ix.ctypes.data_as(C.c_void_p), bits)


@pytest.mark.parametrize("bits", [32, 64])
def test_csr_validation(bits):
    ok = _validate(3, 5, [0, 2, 2, 4], [0, 4, 1, 3], bits)
    assert ok == 0
    assert _validate(3, 5, [1, 2, 2, 4], [0, 4, 1, 3], bits) == 2          # indptr[0] != 0
    assert _validate(3, 5, [0, 3, 2, 4], [0, 4, 1, 3], bits) == 2          # decreasing
    assert _validate(3, 5, [0, 2, 2, 3], [0, 4, 1, 3], bits) == 2          # indptr[N] != nnz
    assert _validate(3, 5, [0, 2, 2, 4], [0, 5, 1, 3], bits) == 2          # index >= K
    assert _validate(3, 5, [0, 2, 2, 4], [0, -1, 1, 3], bits) == 2         # negative index
    assert "out of range" in _abi.last_error()
    assert _validate(0, 5, [0], [], bits) == 0                             # empty matrix
    assert _validate(2, 0, [0, 0, 0], [], bits) == 0                       # K = 0, no nonzeros


def test_struct_layouts_match_header(tmp_path):
    """pfrt_peer_set and pfrt_ipc_handle as the C compiler lays them out equal
    the ctypes mirrors the Python wrapper passes."""
    src = tmp_path / "layout.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "pfrt_cuda.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(pfrt_peer_set),'
                   ' offsetof(pfrt_peer_set, world), offsetof(pfrt_peer_set, y),'
                   ' offsetof(pfrt_peer_set, recv), offsetof(pfrt_peer_set, state),'
                   ' offsetof(pfrt_peer_set, ns), offsetof(pfrt_peer_set, max_m),'
                   ' offsetof(pfrt_peer_set, y_peer), offsetof(pfrt_peer_set, sig),'
                   ' sizeof(pfrt_ipc_handle)); return 0;}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    P = _abi.PeerSet
    assert got == [C.sizeof(P), P.world.offset, P.y.offset, P.recv.offset, P.state.offset, P.ns.offset,
                   P.max_m.offset, P.y_peer.offset, P.sig.offset, C.sizeof(_abi.IpcHandle)]


@pytest.mark.parametrize("name", ["libpfrt_cuda.so", "libpfrt_cuda_backend.so", "libpfrt_session.so"])
def test_libraries_share_the_system_libstdcxx(name):
    """Each library links the shared libstdc++ and exports none of its
    internals.  These libraries are loaded into processes that hold the
    system's libstdc++ already (Python, the PyFlameRT runtime); a library with
    its own static copy of the iostream and locale code broke std::ostringstream
    across the library boundary (a null facet when the plugin formatted a
    number in a Python process)."""
    path = os.path.join(ROOT, "pyflamert_b200", "lib", name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not built")
    needed = subprocess.run(["readelf", "-d", path], capture_output=True, text=True, check=True).stdout
    assert "libstdc++.so.6" in needed
    syms = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    leaked = [l for l in syms.splitlines() if "_ZNSo" in l or "codecvt" in l or "_ZNSt6locale" in l]
    assert not leaked, leaked[:5]
