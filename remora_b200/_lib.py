"""ctypes binding of libremora_b200.so (the C ABI in include/remora_b200.h).

Loading fails loudly: there is no CPU fallback.  Set REMORA_B200_LIB to use a
library outside the package directory.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

from remora_b200.errors import (
    CUDAError,
    RemoraB200Error,
    RemoraLimitError,
    RemoraShapeError,
    RemoraTimeoutError,
    RemoraUnsupportedError,
)

# ---------------------------------------------------------------- constants
MAX_RANK = 10
F32, I32, BOOL = 0, 1, 2

OK = 0
ERR_RANK = -1
ERR_SHAPE = -2
ERR_UNSUPPORTED = -3
ERR_CUDA = -4
ERR_ARG = -5
ERR_TIMEOUT = -6
ERR_JIT = -7
ERR_LIMIT = -8

(OP_INPUT, OP_CONST, OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_LT, OP_LE, OP_GT, OP_GE,
 OP_EQ, OP_NE, OP_SELECT, OP_AND, OP_OR, OP_NEG, OP_EXP, OP_LOG, OP_SQRT) = range(19)

MAP_MAX_INSTR = 48
MAP_MAX_INPUTS = 8
MAP_MAX_REGS = 64

FOLD_ADD, FOLD_MUL = 0, 1
FOLD_CELL, FOLD_ALL = 0, 1
EPI_NONE, EPI_SQRT = 0, 1
PREC_TF32, PREC_3XTF32, PREC_2XTF32 = 0, 1, 2


# ----------------------------------------------------------------- structs
class RemoraMapInstr(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.c_uint8),
        ("dst", ctypes.c_uint8),
        ("a", ctypes.c_uint8),
        ("b", ctypes.c_uint8),
        ("c", ctypes.c_uint8),
        ("pad_", ctypes.c_uint8 * 3),
        ("imm_f", ctypes.c_float),
        ("imm_i", ctypes.c_int32),
    ]


class RemoraMapProgram(ctypes.Structure):
    _fields_ = [
        ("n_instr", ctypes.c_int32),
        ("n_inputs", ctypes.c_int32),
        ("compute_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("result", ctypes.c_int32),
        ("in_dtype", ctypes.c_int32 * MAP_MAX_INPUTS),
        ("code", RemoraMapInstr * MAP_MAX_INSTR),
    ]


class RemoraFoldSpec(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.c_int32),
        ("mode", ctypes.c_int32),
        ("cell_rank", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("epilogue", ctypes.c_int32),
        ("has_premap", ctypes.c_int32),
        ("init_f", ctypes.c_float),
        ("init_i", ctypes.c_int32),
        ("premap", RemoraMapProgram),
    ]


class RemoraScanSpec(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("exclusive", ctypes.c_int32),
        ("right", ctypes.c_int32),
        ("init_f", ctypes.c_float),
        ("init_i", ctypes.c_int32),
    ]


class RemoraGemmSpec(ctypes.Structure):
    _fields_ = [("precision", ctypes.c_int32), ("reserved_", ctypes.c_int32)]


class RemoraConvSpec(ctypes.Structure):
    _fields_ = [
        ("stride", ctypes.c_int32),
        ("pad", ctypes.c_int32),
        ("precision", ctypes.c_int32),
        ("reserved_", ctypes.c_int32),
    ]


class RemoraIm2colSpec(ctypes.Structure):
    _fields_ = [
        ("kh", ctypes.c_int32),
        ("kw", ctypes.c_int32),
        ("stride", ctypes.c_int32),
        ("reserved_", ctypes.c_int32),
    ]


class RemoraFilterPred(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.c_int32),
        ("lit_f", ctypes.c_float),
        ("lit_i", ctypes.c_int32),
        ("reserved_", ctypes.c_int32),
    ]


# ------------------------------------------------------------------ loading
_VP = ctypes.c_void_p
_I32 = ctypes.c_int32
_SZ = ctypes.c_size_t
_PROTOTYPES: dict[str, tuple] = {
    "remora_b200_init": (_I32, [ctypes.c_int, ctypes.POINTER(_VP)]),
    "remora_b200_shutdown": (_I32, [_VP]),
    "remora_b200_last_error": (_I32, [ctypes.c_char_p, _SZ]),
    "remora_b200_version": (ctypes.c_char_p, []),
    "remora_b200_launch_count": (ctypes.c_ulonglong, []),
    "remora_b200_malloc": (_I32, [_VP, _SZ, ctypes.POINTER(_VP)]),
    "remora_b200_free": (_I32, [_VP, _VP]),
    "remora_b200_memcpy_h2d": (_I32, [_VP, _VP, _VP, _SZ, _VP]),
    "remora_b200_memcpy_d2h": (_I32, [_VP, _VP, _VP, _SZ, _VP]),
    "remora_b200_memset_d32": (_I32, [_VP, _VP, ctypes.c_uint32, _SZ, _VP]),
    "remora_b200_synchronize": (_I32, [_VP, _VP]),
    "remora_b200_wait_check": (_I32, [_VP, ctypes.c_int64, _I32, _VP]),
    "remora_b200_set_persistent_sms": (_I32, [_VP, _I32]),
    "remora_b200_host_register": (_I32, [_VP, _SZ]),
    "remora_b200_host_unregister": (_I32, [_VP]),
    "remora_b200_jit_check": (_I32, [ctypes.POINTER(RemoraMapProgram), _I32, ctypes.c_char_p, _SZ]),
    "remora_b200_map": (
        _I32,
        [_VP, ctypes.POINTER(RemoraMapProgram), ctypes.POINTER(_VP), ctypes.POINTER(_I32), _I32, _VP, _I32, _VP],
    ),
    "remora_b200_fold": (
        _I32,
        [_VP, ctypes.POINTER(RemoraFoldSpec), ctypes.POINTER(_VP), ctypes.POINTER(_I32), _I32, _VP, _I32, _VP],
    ),
    "remora_b200_array_fold": (_I32, [_VP, ctypes.POINTER(RemoraFoldSpec), _VP, _I32, _VP, _VP, _VP]),
    "remora_b200_scan": (_I32, [_VP, ctypes.POINTER(RemoraScanSpec), _VP, _VP, _I32, _VP]),
    "remora_b200_scan_noalloc": (_I32, [_VP, ctypes.POINTER(RemoraScanSpec), _VP, _VP, _I32, _VP]),
    "remora_b200_gemm": (_I32, [_VP, ctypes.POINTER(RemoraGemmSpec), _VP, _VP, _VP, _I32, _VP]),
    "remora_b200_conv2d_fwd": (_I32, [_VP, ctypes.POINTER(RemoraConvSpec), _VP, _VP, _VP, _VP, _VP]),
    "remora_b200_conv2d_dgrad": (_I32, [_VP, ctypes.POINTER(RemoraConvSpec), _VP, _VP, _VP, _VP]),
    "remora_b200_conv2d_wgrad": (_I32, [_VP, ctypes.POINTER(RemoraConvSpec), _VP, _VP, _VP, _VP]),
    "remora_b200_im2col": (_I32, [_VP, ctypes.POINTER(RemoraIm2colSpec), _VP, _VP, _VP]),
    "remora_b200_col2im": (_I32, [_VP, ctypes.POINTER(RemoraIm2colSpec), _VP, _VP, _VP]),
    "remora_b200_transpose": (_I32, [_VP, _I32, _VP, _VP, _VP]),
    "remora_b200_sort": (_I32, [_VP, _I32, _VP, _VP, _I32, _VP]),
    "remora_b200_grade": (_I32, [_VP, _I32, _VP, _VP, _I32, _VP]),
    "remora_b200_filter": (_I32, [_VP, _I32, _VP, _VP, _I32, ctypes.POINTER(RemoraFilterPred), _VP, _VP, _VP]),
    "remora_b200_replicate": (_I32, [_VP, _I32, _VP, _VP, _VP, _VP, _VP]),
    "remora_b200_rotate": (_I32, [_VP, _I32, ctypes.c_int64, _VP, _VP, _I32, _VP]),
    "remora_b200_append": (_I32, [_VP, _I32, _VP, _VP, _VP, _I32, _VP]),
}

_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    env = os.environ.get("REMORA_B200_LIB")
    if env:
        return Path(env)
    return Path(__file__).resolve().parent / "libremora_b200.so"


def lib() -> ctypes.CDLL:
    """Return the loaded library, loading it on first use (raises if absent)."""
    global _lib
    if _lib is None:
        path = library_path()
        if not path.exists():
            raise RemoraB200Error(
                f"{path} is not built; run `python -m remora_b200.csrc.build` "
                "(there is no CPU fallback for the B200 backend)"
            )
        handle = ctypes.CDLL(str(path))
        for name, (restype, argtypes) in _PROTOTYPES.items():
            fn = getattr(handle, name, None)
            if fn is None:
                continue
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    """Names of the C-ABI entry points the loaded library exports."""
    handle = lib()
    return [name for name in _PROTOTYPES if hasattr(handle, name)]


def launch_count() -> int:
    """Kernels the library has enqueued in this process so far (launched, or
    recorded into a CUDA graph under stream capture)."""
    return int(lib().remora_b200_launch_count())


def last_error() -> str:
    buf = ctypes.create_string_buffer(2048)
    lib().remora_b200_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


_ERRORS = {
    ERR_RANK: RemoraShapeError,
    ERR_SHAPE: RemoraShapeError,
    ERR_UNSUPPORTED: RemoraUnsupportedError,
    ERR_CUDA: CUDAError,
    ERR_ARG: RemoraB200Error,
    ERR_TIMEOUT: RemoraTimeoutError,
    ERR_JIT: RemoraB200Error,
    ERR_LIMIT: RemoraLimitError,
}


def check(status: int, what: str = "") -> None:
    """Raise the exception matching a C-ABI status code."""
    if status == OK:
        return
    cls = _ERRORS.get(status, RemoraB200Error)
    msg = last_error()
    raise cls(f"{what}: {msg} (status {status})" if what else f"{msg} (status {status})")
