"""ctypes binding of the C ABI declared in ``include/g4b.h``.

The library is ``libg4b.so`` next to this file, built in-tree by
``g4b._build``.  If it is missing it is built on first use when nvcc is
available; otherwise loading fails loudly -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

from . import _build

# status codes (include/g4b.h)
G4B_OK = 0
G4B_E_SHAPE = -1
G4B_E_ALIGN = -2
G4B_E_ARCH = -3
G4B_E_CUDA = -4
G4B_E_FAULT_INJECTED = -5
G4B_E_ARG = -6
G4B_E_WORKSPACE = -7
G4B_E_TIMEOUT = -8

GEMV_PDL = 1
CHAIN_ALLREDUCE = 1
CHAIN_RUN_PDL = 1
GEMM_PDL = 1
DT_F32 = 0
DT_F16 = 1
SCALE_F16 = 0
SCALE_E4M3 = 1

Q_VERSION = 0
Q_DEVICE_OK = 1
Q_SM_COUNT = 2
Q_LAUNCHES = 3
Q_FAULT_COUNTER = 4
Q_KERNEL_STATUS = 5

_STATUS_NAMES = {
    G4B_E_SHAPE: "G4B_E_SHAPE", G4B_E_ALIGN: "G4B_E_ALIGN", G4B_E_ARCH: "G4B_E_ARCH",
    G4B_E_CUDA: "G4B_E_CUDA", G4B_E_FAULT_INJECTED: "G4B_E_FAULT_INJECTED", G4B_E_ARG: "G4B_E_ARG",
    G4B_E_WORKSPACE: "G4B_E_WORKSPACE", G4B_E_TIMEOUT: "G4B_E_TIMEOUT",
}

# The entry points declared in include/g4b.h: name -> (restype, argtypes)
_P = C.c_void_p
_I = C.c_int
_F = C.c_float
_Z = C.c_size_t
class GemmSeg(C.Structure):
    """g4b_gemm_seg: one weight of g4b_gemm_i4_fused."""
    _fields_ = [("wp", C.c_void_p), ("scales_f16", C.c_void_p), ("y", C.c_void_p), ("N", C.c_int)]


SIGNATURES = {
    "g4b_last_error": (C.c_char_p, []),
    "g4b_version": (_I, []),
    "g4b_query": (C.c_longlong, [_I]),
    "g4b_stream_wait": (_I, [_P, _I]),
    "g4b_gemv_workspace_bytes": (_Z, [_I, _I, _I, _I]),
    "g4b_gemv_i4": (_I, [_P, _I, _I, _P, _P, _I, _F, _P, _I, _I, _I, _I, _P, _Z, _P]),
    "g4b_gemv_i4_ex": (_I, [_P, _I, _I, _P, _P, _I, _F, _P, _I, _I, _I, _I, _P, _Z, C.c_uint, _P]),
    "g4b_gemv_i4_noalloc": (_I, [_P, _I, _I, _P, _P, _I, _F, _P, _I, _I, _I, _I, _P]),
    "g4b_gemv_fused_workspace_bytes": (_Z, [_I, _P, _I]),
    "g4b_gemv_i4_fused": (_I, [_P, _I, _I, _P, _I, _I, _I, _P, _Z, C.c_uint, _P]),
    "g4b_reduce_partials": (_I, [_P, _P, _I, _I, _P]),
    "g4b_dequant_i4": (_I, [_P, _P, _I, _F, _P, _I, _I, _I, _P]),
    "g4b_cast": (_I, [_P, _I, _P, _I, _Z, _P]),
    "g4b_cast_i8": (_I, [_P, _I, _P, _P, _I, _I, _P]),
    "g4b_quant_i4": (_I, [_P, _I, _I, _P, _P, _P, _P, _P]),
    "g4b_quant_e4m3": (_I, [_P, _I, _I, _I, _P, _P]),
    "g4b_quant_w8a8": (_I, [_P, _P, _I, _I, _P, _P, _P, _P, _P]),
    "g4b_gemm_i4_workspace_bytes": (_Z, [_I, _I, _I, _I]),
    "g4b_gemm_i4": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _P, _Z, _P]),
    "g4b_gemm_i4_ex": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _P, _Z, C.c_uint, _P]),
    "g4b_gemm_i4_fused": (_I, [_P, _I, _I, _I, _P, _I, _I, _P, _Z, C.c_uint, _P]),
    "g4b_allreduce_buffer_bytes": (_Z, [_I, _I]),
    "g4b_allreduce_f32": (_I, [_P, _P, _I, _I, _I, _P, _P, C.c_uint, _P]),
    "g4b_comm_alloc": (_I, [_Z, C.POINTER(_P)]),
    "g4b_comm_free": (_I, [_P]),
    "g4b_ipc_handle": (_I, [_P, _P]),
    "g4b_ipc_open": (_I, [_P, C.POINTER(_P)]),
    "g4b_ipc_close": (_I, [_P]),
    "g4b_gemm_w8a8": (_I, [_P, _P, _P, _P, _P, _I, _P, _I, _I, _I, _P]),
    "g4b_gemm_w4a8": (_I, [_P, _P, _P, _P, _P, _P, _I, _P, _I, _I, _I, _P]),
    "g4b_gemv_chain_create": (_I, [_P, _I, _I, _I, _I, C.POINTER(_P)]),
    "g4b_gemv_chain_exchange_bytes": (_Z, [_P, _I, _I]),
    "g4b_gemv_chain_create_tp": (_I, [_P, _I, _I, _I, _I, _P, _I, _I, _Z, C.POINTER(_P)]),
    "g4b_gemv_chain_create_fused": (_I, [_P, _P, _I, _I, _I, _I, C.POINTER(_P)]),
    "g4b_attn_prepkv": (_I, [_P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "g4b_attn_workspace_bytes": (_Z, [_I, _I, _I, _I]),
    "g4b_attn_decode": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P, _Z, _P]),
    "g4b_attn_decode_prepkv": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I,
                                    _P, _P, _Z, _P]),
    "g4b_rows_rmsnorm": (_I, [_P, _I, _P, _P, _I, _I, _I, _P]),
    "g4b_rows_normadd": (_I, [_P, _I, _P, _P, _I, _I, _F, _P]),
    "g4b_gelumul": (_I, [_P, _P, _I, _P, _I, _Z, _P]),
    "g4b_attn_prefill_prepkv": (_I, [_P, _P, _I, _I, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "g4b_attn_prefill": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "g4b_gemv_chain_workspace_bytes": (_Z, [_P]),
    "g4b_gemv_chain_plan": (_I, [_P, _P, _I, _I, _I, _P]),
    "g4b_gemv_chain_run": (_I, [_P, _P, _Z, _P]),
    "g4b_gemv_chain_run_ex": (_I, [_P, _P, _Z, C.c_uint, _P]),
    "g4b_gemv_chain_destroy": (None, [_P]),
}


class GemvSegment(C.Structure):
    """struct g4b_gemv_segment (include/g4b.h)."""
    _fields_ = [("wp", C.c_void_p), ("scales", C.c_void_p), ("inv", C.c_float), ("y", C.c_void_p), ("N", C.c_int)]


class GemvChainStep(C.Structure):
    """struct g4b_gemv_chain_step (include/g4b.h)."""
    _fields_ = [("x", C.c_void_p), ("K", C.c_int), ("nseg", C.c_int), ("seg", GemvSegment * 3),
                ("flags", C.c_uint)]


XF_NONE = 0
XF_RMSNORM = 1
XF_NORMADD = 2
XF_GELU_MUL = 3


class ChainXform(C.Structure):
    """struct g4b_chain_xform (include/g4b.h)."""
    _fields_ = [("kind", C.c_int), ("a", C.c_void_p), ("b", C.c_void_p), ("w", C.c_void_p), ("w_post", C.c_void_p),
                ("h_out", C.c_void_p), ("scale", C.c_float), ("eps", C.c_float)]


class ChainStepPlan(C.Structure):
    """struct g4b_chain_step_plan (include/g4b.h)."""
    _fields_ = [("x_forwarded", C.c_int), ("wait_from", C.c_int), ("x_early", C.c_int), ("reserved", C.c_int)]


class G4BError(RuntimeError):
    """A g4b entry point returned a negative status."""

    def __init__(self, op: str, code: int, msg: str):
        super().__init__(f"{op} failed with {_STATUS_NAMES.get(code, code)}: {msg}")
        self.op = op
        self.code = code


_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return _build.LIB_PATH


def load(build_if_missing: bool = True):
    """Load (building if needed) the CUDA library and bind its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB_PATH
        if not os.path.exists(path) or (build_if_missing and not _build.up_to_date()
                                        and _nvcc_available()):
            if not build_if_missing:
                raise ImportError(f"g4b CUDA library not built: {path} is missing")
            _build.build()
        L = C.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _nvcc_available() -> bool:
    try:
        _build.nvcc_path()
        return True
    except RuntimeError:
        return False


def last_error() -> str:
    return load().g4b_last_error().decode(errors="replace")


def check(op: str, status: int) -> None:
    if status != G4B_OK:
        raise G4BError(op, status, last_error())


def query(what: int) -> int:
    return int(load().g4b_query(what))


def launches() -> int:
    """Kernels launched through the library by this process so far."""
    return query(Q_LAUNCHES)
