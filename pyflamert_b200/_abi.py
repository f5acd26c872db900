"""ctypes prototypes of the C ABI declared in include/pfrt_cuda.h."""
from __future__ import annotations

import ctypes as C
import os
import threading

PFRT_OUT_F32, PFRT_OUT_S8, PFRT_OUT_U8 = 0, 1, 2

STATUS_NAMES = {
    0: "PFRT_OK", 1: "PFRT_ERR_INVALID_ARGUMENT", 2: "PFRT_ERR_BAD_CSR", 3: "PFRT_ERR_CUDA",
    4: "PFRT_ERR_OUT_OF_MEMORY", 5: "PFRT_ERR_UNSUPPORTED", 6: "PFRT_ERR_DEVICE_TIMEOUT",
    7: "PFRT_ERR_NO_DEVICE",
}

_P, _I64, _I32, _F32, _INT, _SZ = C.c_void_p, C.c_int64, C.c_int32, C.c_float, C.c_int, C.c_size_t

PFRT_MAX_PEERS = 8


class IpcHandle(C.Structure):
    """pfrt_ipc_handle: 64 opaque bytes."""
    _fields_ = [("bytes", C.c_ubyte * 64)]


PFRT_PEER_SIG_WORDS = 16


class PeerSet(C.Structure):
    """pfrt_peer_set (include/pfrt_cuda.h)."""
    _fields_ = [("rank", C.c_int32), ("world", C.c_int32), ("y", C.c_void_p),
                ("recv", C.c_void_p * PFRT_MAX_PEERS), ("state", C.c_void_p),
                ("ns", C.c_int64), ("max_m", C.c_int64),
                ("y_peer", C.c_void_p * PFRT_MAX_PEERS), ("sig", C.c_void_p * PFRT_MAX_PEERS)]


# name -> argument types; every function returns pfrt_status (int) unless listed in _RESTYPE.
PROTOTYPES = {
    "pfrt_version": [],
    "pfrt_last_error": [],
    "pfrt_device_count": [_P],
    "pfrt_ctx_create": [_INT, _P],
    "pfrt_ctx_destroy": [_P],
    "pfrt_ctx_stream": [_P, _P],
    "pfrt_ctx_num_sms": [_P, _P],
    "pfrt_ctx_check": [_P, _P],
    "pfrt_malloc": [_P, _SZ, _P],
    "pfrt_free": [_P, _P],
    "pfrt_host_alloc": [_P, _SZ, _P],
    "pfrt_host_free": [_P, _P],
    "pfrt_memcpy_h2d": [_P, _P, _P, _SZ, _P],
    "pfrt_memcpy_d2h": [_P, _P, _P, _SZ, _P],
    "pfrt_memcpy_d2d": [_P, _P, _P, _SZ, _P],
    "pfrt_memset": [_P, _P, _INT, _SZ, _P],
    "pfrt_memcpy_h2d_staged": [_P, _P, _P, _SZ, _P],
    "pfrt_memcpy_d2h_staged": [_P, _P, _P, _SZ, _P],
    "pfrt_fweight_create": [_P, _I64, _I64, _INT, _P, _P],
    "pfrt_fweight_destroy": [_P],
    "pfrt_gemm_f32": [_P, _I64, _INT, _F32, _P, _P, _F32, _P, _I64, _P, _P],
    "pfrt_gemm_f32_noalloc": [_P, _I64, _INT, _F32, _P, _P, _F32, _P, _I64, _P, _P],
    "pfrt_gemm_f32_dense": [_P, _I64, _I64, _I64, _INT, _INT, _F32, _P, _P, _F32, _P, _I64, _P, _P],
    "pfrt_qweight_create": [_P, _I64, _I64, _P, _I32, _P, _I64, _P],
    "pfrt_qweight_destroy": [_P],
    "pfrt_qlinear": [_P, _P, _I64, _P, _I64, _INT, _F32, _I32, _P, _INT, _INT, _F32, _I32, _P, _I64, _P, _P],
    "pfrt_qlinear_host": [_P, _P, _I64, _P, _I64, _INT, _F32, _I32, _P, _INT, _INT, _F32, _I32, _P, _I64, _P],
    "pfrt_csr_create": [_P, _I64, _I64, _I64, _P, _P, _INT, _P, _P],
    "pfrt_csr_destroy": [_P],
    "pfrt_csr_validate_host": [_I64, _I64, _I64, _P, _P, _INT],
    "pfrt_csr_info": [_P, _P, _P, _P],
    "pfrt_spmm": [_P, _P, _I64, _P, _I64, _P, _I64, _P],
    "pfrt_spmm_csr_f32": [_P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _P, _I64, _P],
    "pfrt_csr_from_magnitude_pruning": [_P, _I64, _I64, _P, _F32, _P, _P],
    "pfrt_csr_from_nm_pruning": [_P, _I64, _I64, _P, _I32, _I32, _P, _P],
    "pfrt_ipc_get_handle": [_P, _P, _P],
    "pfrt_ipc_open": [_P, _P, _P],
    "pfrt_ipc_close": [_P, _P],
    "pfrt_spmm_allgather": [_P, _P, _I64, _P, _I64, _P, _P],
    "pfrt_peer_allgather": [_P, _I64, _P, _P],
    "pfrt_peer_reset": [_P, _P, _P],
    "pfrt_quantize_f32": [_P, _I64, _P, _F32, _I32, _INT, _P, _P],
    "pfrt_add_rowvec_f32": [_P, _I64, _I64, _P, _P, _P, _P],
    "pfrt_relu_f32": [_P, _I64, _P, _P, _P],
}
_RESTYPE = {"pfrt_version": C.c_char_p, "pfrt_last_error": C.c_char_p}

_LIB = None
_LOCK = threading.Lock()


class PfrtError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def lib_path() -> str:
    return os.environ.get(
        "PFRT_CUDA_LIB",
        os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libpfrt_cuda.so"))


def lib():
    """The loaded C ABI library.  Raises if it has not been built."""
    global _LIB
    if _LIB is None:
        with _LOCK:
            if _LIB is None:
                path = lib_path()
                if not os.path.exists(path):
                    raise RuntimeError(
                        f"libpfrt_cuda.so not found at {path}; build it with "
                        f"`python -m pyflamert_b200.build` (no CPU fallback exists)")
                L = C.CDLL(path)
                for name, args in PROTOTYPES.items():
                    f = getattr(L, name)
                    f.argtypes = args
                    f.restype = _RESTYPE.get(name, C.c_int)
                _LIB = L
    return _LIB


def last_error() -> str:
    return lib().pfrt_last_error().decode()


def check(st: int, what: str = "") -> None:
    if st != 0:
        msg = last_error()
        raise PfrtError(st, f"{what}: {msg}" if what else msg)
