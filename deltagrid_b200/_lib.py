"""ctypes binding of libdeltagrid_b200.so (the C ABI declared in include/deltagrid_b200.h).

The library is built in-tree by ``python -m deltagrid_b200.build``.  There is
no fallback: if the library is missing or fails to load, every entry point
raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdeltagrid_b200.so")

DTYPE_F32, DTYPE_F64, DTYPE_F16, DTYPE_BF16 = 0, 1, 2, 3
ALGO_AUTO, ALGO_SEQUENTIAL, ALGO_CHUNKED_TC, ALGO_CHUNKED_TC_ROWS = 0, 1, 2, 3
PKM_AUTO, PKM_ONE_STEP, PKM_PIPELINED, PKM_WARP_SPECIALIZED = 0, 1, 2, 3
DEVCHK_INDEX_RANGE = 0x1

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t

# name -> argtypes (restype is int status unless listed in _RESTYPE)
_SIGS = {
    "dg_status_string": [_I],
    "dg_abi_version": [],
    "dg_last_cuda_error": [],
    "dg_dense_forward": [_I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P],
    "dg_dense_forward_ex": [_I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I, _P],
    "dg_dense_forward_ex2": [_I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _I, _P],
    "dg_set_wait_limit": [ctypes.c_uint],
    "dg_dense_step": [_I, _I, _I, _I, _I, _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,
                      _P, _I, _I64, _I64, _P, _P, _P, _P],
    "dg_pkm_forward": [_I, _I, _I, _I, _I, _I64, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P],
    "dg_pkm_forward_ex": [_I, _I, _I, _I, _I, _I64, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _I, _P, _SZ,
                          _P],
    "dg_pkm_forward_workspace_size": [_I, _I, _I, _I, _I, _I64, _I, _I],
    "dg_pkm_forward_noalloc": [_I, _I, _I, _I, _I, _I64, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P],
    "dg_pkm_step": [_I, _I, _I, _I, _I64, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P],
    "dg_read_device_status": [_P, _I, _P, _P],
    "dg_pkm_route": [_I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    "dg_dense_route": [_I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    "dg_fxp_dense_forward": [_I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P],
    "dg_fxp_pkm_forward": [_I, _I, _I, _I64, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    "dg_dense_backward_workspace_size": [_I, _I, _I, _I],
    "dg_dense_backward": [_I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P,
                          _P, _P],
    "dg_pkm_backward": [_I, _I, _I, _I, _I, _I64, _I, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P,
                        _P, _P],
}
_RESTYPE = {"dg_status_string": ctypes.c_char_p, "dg_set_wait_limit": ctypes.c_uint, "dg_pkm_forward_workspace_size": ctypes.c_size_t,
            "dg_dense_backward_workspace_size": ctypes.c_size_t}

_lib = None
_lock = threading.Lock()


class DeltaGridError(RuntimeError):
    """A C-ABI call returned a non-zero dg_status."""


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"deltagrid_b200 native library not found at {LIB_PATH}; "
                        "build it with `python -m deltagrid_b200.build`")
                L = ctypes.CDLL(LIB_PATH)
                for name, args in _SIGS.items():
                    if not hasattr(L, name):
                        continue
                    fn = getattr(L, name)
                    fn.argtypes = args
                    fn.restype = _RESTYPE.get(name, ctypes.c_int)
                _lib = L
    return _lib


def has_symbol(name: str) -> bool:
    return hasattr(lib(), name)


def check(status: int, what: str) -> None:
    if status != 0:
        L = lib()
        msg = L.dg_status_string(status).decode()
        if status == -5:
            msg += f" (cudaError {L.dg_last_cuda_error()})"
        raise DeltaGridError(f"{what} failed: {msg} [status {status}]")


_fns = {}


def fn(name: str):
    """The bound C function `name` (looked up once)."""
    f = _fns.get(name)
    if f is None:
        f = getattr(lib(), name)
        _fns[name] = f
    return f


def call(name: str, *args) -> None:
    check(fn(name)(*args), name)
