"""ctypes binding of libawq_b200.so (declarations: include/awq_b200.h).

The library is built in-tree by ``make -C qwen2-7b-triton_engine_b200`` (or
``__graft_entry__.build()``).  Loading fails loudly when it is missing: there is no
CPU or eager-PyTorch fallback behind these functions.
"""
from __future__ import annotations

import ctypes
import os
import pathlib

PKG_ROOT = pathlib.Path(__file__).resolve().parent.parent
LIB_PATH = pathlib.Path(os.environ.get("AWQ_B200_LIB", PKG_ROOT / "lib" / "libawq_b200.so"))

AWQ_OK = 0
AWQ_ERR_INVALID_ARG = -1
AWQ_ERR_UNSUPPORTED = -2
AWQ_ERR_CUDA = -3
AWQ_ERR_WORKSPACE = -4
AWQ_ERR_DEVICE = -5

AWQ_PATH_AUTO = 0
AWQ_PATH_DECODE = 1
AWQ_PATH_TC = 2
AWQ_PATH_TS = 3

# Every symbol include/awq_b200.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_INT = ctypes.c_int
SIGNATURES = {
    "awq_version": ([], _INT),
    "awq_last_error": ([], ctypes.c_char_p),
    "awq_dequant_f16": ([_P, _P, _P, _P, _I64, _I64, _I64, _P], _INT),
    "awq_gemm_workspace_bytes": ([_I64, _I64, _I64, _I64], _SZ),
    "awq_workspace_init": ([_P, _SZ, _P], _INT),
    "awq_gemm_f16": ([_P, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _SZ, _P], _INT),
    "awq_gemm_f16_ex": ([_P, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _SZ, _P,
                         _INT], _INT),
    "awq_gemm_f16_noalloc": ([_P, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P], _INT),
    "awq_gemm_f16_bias": ([_P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _SZ,
                           _P], _INT),
    "awq_tc_supported": ([_P, _I64, _P, _P, _P, _I64, _I64, _I64, _I64], _INT),
    "awq_tc_schedule": ([_I64, _I64, _I64, _INT, _P, _P], _INT),
    "awq_device_status": ([_P, ctypes.POINTER(ctypes.c_int)], _INT),
    "awq_tp_comm_create": ([_INT, _INT, _I64, _P, ctypes.POINTER(_P)], _INT),
    "awq_tp_comm_create_ex": ([_INT, _INT, _I64, _I64, _P, ctypes.POINTER(_P)], _INT),
    "awq_tp_comm_open": ([_P, _P], _INT),
    "awq_tp_comm_set_timeout": ([_P, ctypes.c_uint64], _INT),
    "awq_tp_comm_reset": ([_P], _INT),
    "awq_tp_comm_destroy": ([_P], _INT),
    "awq_allreduce_supported": ([_P, _P, _I64, _P, _I64, _I64, _I64, _I64], _INT),
    "awq_gemm_f16_allreduce": ([_P, _P, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P,
                                _SZ, _P], _INT),
    "awq_gemm_silu_mul_workspace_bytes": ([_I64, _I64, _I64, _I64], _SZ),
    "awq_gemm_f16_silu_mul": ([_P, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _SZ,
                               _P], _INT),
}

AWQ_IPC_HANDLE_BYTES = 64
AWQ_MAX_WORLD = 8
# bits of the device status word (awq_device_status)
STATUS_BARRIER_TIMEOUT = 1
STATUS_SHAPE = 2
STATUS_PEER_TIMEOUT = 4

_lib = None


class AwqError(RuntimeError):
    """A non-zero return code from libawq_b200."""

    def __init__(self, code: int, message: str):
        super().__init__(f"libawq_b200 error {code}: {message}")
        self.code = code


def load() -> ctypes.CDLL:
    """Open the shared library once and attach the signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing; build it with `make -C {PKG_ROOT}` "
            "(the AWQ path has no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != AWQ_OK:
        msg = load().awq_last_error()
        raise AwqError(rc, msg.decode() if msg else "")
