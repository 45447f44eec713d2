"""ctypes binding of libdsv32_int8.so (the C ABI in include/dsv32_int8.h).

The library is loaded from the package directory only; there is no fallback. Importing this
module does not need a GPU; calling a kernel entry point does (the library returns
DSV32_ERR_NO_DEVICE otherwise, surfaced as RuntimeError).
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

DSV32_OK = 0
DSV32_ERR_INVALID_ARG = 1
DSV32_ERR_UNSUPPORTED = 2
DSV32_ERR_CUDA = 3
DSV32_ERR_DEVICE_TIMEOUT = 4
DSV32_ERR_NO_DEVICE = 5

DSV32_F32 = 0
DSV32_BF16 = 1
DSV32_F16 = 2

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int

# name -> (restype, argtypes); mirrors include/dsv32_int8.h
SIGNATURES = {
    "dsv32_act_quant": (_i32, [_p, _i32, _i64, _i64, _i32, _p, _p, _p]),
    "dsv32_int8_gemm": (_i32, [_p, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _p, _i64, _p]),
    "dsv32_int8_gemm_workspace_bytes": (_i64, [_i64, _i64, _i64]),
    "dsv32_int8_gemm_noalloc": (_i32, [_p, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _p]),
    "dsv32_int8_gemm_partials": (_i32, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _p, _i64, _p]),
    "dsv32_int8_index": (_i32, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _i64, _i64, _p]),
    "dsv32_topk_workspace_bytes": (_i64, [_i64, _i64, _i64, _i32]),
    "dsv32_topk": (_i32, [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _p, _p, _i64, _p]),
    "dsv32_int8_index_topk": (_i32, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _i64, _i64, _i32,
                                     _i64, _i64, _p, _p, _p, _i64, _p]),
    "dsv32_rotate_quant": (_i32, [_p, _i32, _i64, _i32, _p, _p, _p, _p]),
    "dsv32_weight_quant": (_i32, [_p, _i32, _i64, _i64, _p, _p, _p]),
    "dsv32_device_status": (_i32, [_i32, ctypes.POINTER(ctypes.c_uint32)]),
    "dsv32_set_wait_limit": (_i32, [_i64]),
    "dsv32_status_string": (ctypes.c_char_p, [_i32]),
    "dsv32_last_error_message": (ctypes.c_char_p, []),
    "dsv32_topk_parts": (_i32, [ctypes.POINTER(_p), ctypes.POINTER(_p), _i32, _i64, _i64, _i64, _i64, _p, _p, _p,
                                _i64, _p]),
    "dsv32_topk_parts_to": (_i32, [ctypes.POINTER(_p), ctypes.POINTER(_p), _i32, _i64, _i64, _i64, _i64,
                                   ctypes.POINTER(_p), ctypes.POINTER(_p), _i32, _p, _i64, _p]),
    "dsv32_device_alloc": (_i32, [_i64, ctypes.POINTER(_p)]),
    "dsv32_device_free": (_i32, [_p]),
    "dsv32_copy_async": (_i32, [_p, _p, _i64, _p]),
    "dsv32_ipc_export": (_i32, [_p, _p]),
    "dsv32_ipc_open": (_i32, [_p, ctypes.POINTER(_p)]),
    "dsv32_ipc_close": (_i32, [_p]),
    "dsv32_abi_version": (_i32, []),
}

ABI_VERSION = 7
IPC_HANDLE_BYTES = 64

_LIB = None


def lib_path() -> str:
    return _build.LIB_PATH


def load(build_if_missing: bool = True):
    """Load (building first if needed and allowed) and return the ctypes library."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = lib_path()
    if not os.path.exists(path) or (build_if_missing and _build.needs_build()):
        if not build_if_missing:
            raise RuntimeError(f"{path} is missing; run `python -m deepseek_v32_gtx1650_b200.build`")
        _build.build()
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


class Dsv32Error(RuntimeError):
    def __init__(self, status: int, where: str):
        lib = load()
        msg = lib.dsv32_status_string(status).decode()
        detail = lib.dsv32_last_error_message().decode()
        show = detail and status in (DSV32_ERR_CUDA, DSV32_ERR_UNSUPPORTED)
        super().__init__(f"{where}: {msg}" + (f" ({detail})" if show else ""))
        self.status = status


def check(status: int, where: str) -> None:
    if status != DSV32_OK:
        raise Dsv32Error(status, where)


def device_status(device: int = 0) -> int:
    """Synchronise `device` and return (and clear) the kernels' error word (0 = none). After an
    error the cached GEMM workspaces of the device are dropped (their counters may be stale)."""
    code = ctypes.c_uint32(0)
    st = load().dsv32_device_status(device, ctypes.byref(code))
    if st not in (DSV32_OK, DSV32_ERR_DEVICE_TIMEOUT):
        check(st, "dsv32_device_status")
    if code.value:
        from . import kernels
        for key in [k for k in kernels._GEMM_WS if k[0] == device]:
            del kernels._GEMM_WS[key]
    return int(code.value)
