"""ctypes binding of libflashmlp_b200.so (declared in include/flashmlp_b200.h).

The shared library is the only compute path: if it is missing this module raises, there
is no fallback.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libflashmlp_b200.so")

FMLP_DTYPE_F16 = 0
FMLP_DTYPE_BF16 = 1
FMLP_DTYPE_F32 = 2

FMLP_ACT_LINEAR = 0
FMLP_ACT_LEAKY_RELU = 1
FMLP_ACT_SILU = 2
FMLP_ACT_SIGMOID = 3

FMLP_OK = 0
FMLP_ERR_UNSUPPORTED_D = 3
FMLP_ERR_UNSUPPORTED_E = 4
FMLP_ERR_DEVICE_TIMEOUT = 10
FMLP_ERR_SCRATCH_LIMIT = 11
FMLP_ERR_PEER_ABORT = 12
FMLP_ERR_INVALID_SCALE = 13
FMLP_MAX_PEERS = 8
FMLP_PEER_FLAG_WORDS = 32   # uint32 words of each rank's flag array
FMLP_PEER_STATUS_WORD = 16  # this rank's call status in its own flag array
FMLP_IPC_HANDLE_BYTES = 64

# Every symbol the header declares, with (restype, argtypes).
_c_int, _c_vp, _c_sz, _c_float = ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float
_c_ip = ctypes.POINTER(ctypes.c_int)
SIGNATURES = {
    "fmlp_fwd": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_vp]),
    "fmlp_bwd": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_sz,
         _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_vp],
    ),
    "fmlp_bwd_workspace_size": (_c_sz, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "fmlp_bwd_workspace_size_min": (_c_sz, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "fmlp_bwd_plan": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_sz, _c_ip, _c_ip, _c_ip]),
    "fmlp_bwd_noalloc": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp,
         _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_vp],
    ),
    "fmlp_fwd_shared_x": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_vp]),
    "fmlp_fwd_fp8": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int,
         _c_float, _c_float, _c_float, _c_float, _c_int, _c_int, _c_vp],
    ),
    "fmlp_bwd_shared_x": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_sz,
         _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_vp],
    ),
    "fmlp_bwd_dw_f32": (
        _c_int,
        [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_sz,
         _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_vp],
    ),
    "fmlp_sgd_update": (_c_int, [_c_vp, _c_vp, ctypes.c_longlong, ctypes.c_float, _c_int, _c_vp]),
    "fmlp_grad_allreduce_sgd": (
        _c_int,
        [ctypes.POINTER(_c_vp), ctypes.POINTER(_c_vp), ctypes.POINTER(_c_vp), _c_int, _c_int,
         ctypes.c_longlong, ctypes.c_float, _c_int, ctypes.c_uint, _c_vp],
    ),
    "fmlp_peer_alloc": (_c_int, [_c_sz, ctypes.POINTER(_c_vp)]),
    "fmlp_peer_free": (_c_int, [_c_vp]),
    "fmlp_ipc_get_handle": (_c_int, [_c_vp, _c_vp]),
    "fmlp_ipc_open_handle": (_c_int, [_c_vp, ctypes.POINTER(_c_vp)]),
    "fmlp_ipc_close_handle": (_c_int, [_c_vp]),
    "fmlp_device_status": (_c_int, [_c_int]),
    "fmlp_error_string": (ctypes.c_char_p, [_c_int]),
    "fmlp_abi_version": (_c_int, []),
}

_LIB = None


class FlashMLPError(RuntimeError):
    """A non-zero return code from the C ABI."""

    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: {error_string(code)} (code {code})")


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH.name} is not built; run `python -m flashmlp_b200.build` "
                "(there is no non-CUDA fallback)"
            )
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def error_string(code: int) -> str:
    return lib().fmlp_error_string(code).decode()


def check(code: int, where: str) -> None:
    if code != FMLP_OK:
        raise FlashMLPError(code, where)


def bwd_plan(H: int, B: int, D: int, E: int, dtype_code: int, workspace_bytes: int):
    """(mode, splits, launches) that fmlp_bwd runs for this shape and workspace size on the
    current device: mode 1 = dZ-store, 0 = recompute (fmlp_bwd_plan)."""
    mode, splits, launches = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    check(lib().fmlp_bwd_plan(H, B, D, E, dtype_code, workspace_bytes, ctypes.byref(mode), ctypes.byref(splits),
                              ctypes.byref(launches)), "fmlp_bwd_plan")
    return mode.value, splits.value, launches.value
