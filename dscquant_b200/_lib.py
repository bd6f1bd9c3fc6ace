"""ctypes binding of the C ABI declared in include/dscq_b200.h.

The shared library is built in-tree (dscquant_b200/_native/libdscq_b200.so)
by dscquant_b200.build. There is no fallback: if the library is missing or
the device is not sm_100, calls raise.
"""
from __future__ import annotations

import ctypes
import os
import threading

NATIVE_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_native")
LIB_PATH = os.path.join(NATIVE_DIR, "libdscq_b200.so")

DSCQ_OK, DSCQ_ERR_INVALID, DSCQ_ERR_CUDA, DSCQ_ERR_UNSUPPORTED, DSCQ_ERR_RANGE = 0, 1, 2, 3, 4
BF16, F16, F32 = 0, 1, 2
ACT_SYM, WEIGHT_SYM, ACT_ASYM, ACT_ASYM_TORCH = 0, 1, 2, 3
GEMM_AUTO, GEMM_SMALL_M, GEMM_LARGE_M, GEMM_LARGE_M_DIRECT, GEMM_LARGE_M_PAIR, GEMM_SMALL_M_TC = 0, 1, 2, 3, 4, 5
GEMM_LARGE_M_PAIR_TMEM = 6
QUANT_AUTO, QUANT_TC, QUANT_LEGACY = 0, 1, 2

_i32, _i64, _u32p, _f32, _vp, _cp = (ctypes.c_int, ctypes.c_int64, ctypes.POINTER(ctypes.c_uint32), ctypes.c_float,
                                     ctypes.c_void_p, ctypes.c_char_p)

# name -> (restype, argtypes); kept in the order of include/dscq_b200.h
SIGNATURES = {
    "dscq_version": (_i32, []),
    "dscq_last_error": (_cp, []),
    "dscq_device_status": (_i32, [_i32, _u32p, _i32]),
    "dscq_hadamard": (_i32, [_i32, _vp]),
    "dscq_rotation_split": (_i32, [_i64, ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    "dscq_quantize": (_i32, [_vp, _i32, _i64, _i64, _f32, _i32, _vp, _vp, _vp, _vp]),
    "dscq_rowquant": (_i32, [_vp, _i32, _i64, _i64, _i64, _i32, _i32, _vp, _i32, _f32, _i64, _i64, _vp, _i64, _vp,
                             _vp, _vp, _vp, _i64, _vp]),
    "dscq_rowquant_variant": (_i32, [_vp, _i32, _i64, _i64, _i64, _i32, _i32, _vp, _i32, _f32, _i64, _i64, _vp,
                                     _i64, _vp, _vp, _vp, _vp, _i64, _i32, _vp]),
    "dscq_rowquant_headrot": (_i32, [_vp, _i64, _i64, _i64, _i32, _vp, _vp, _i32, _f32, _i64, _i64, _vp, _i64, _vp,
                                     _vp, _i64, _vp]),
    "dscq_matmul": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp, _vp, _i32, _vp]),
    "dscq_matmul_a8": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp, _vp, _vp]),
    "dscq_matmul_a8_variant": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp, _vp, _i32,
                                      _vp]),
    "dscq_matmul_cols": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32,
                                ctypes.POINTER(ctypes.c_void_p), _i32, _i64, _i64, _i32, _vp]),
    "dscq_rowquant_auto_tc": (_i32, [_i64, _i64]),
    "dscq_scatter_block": (_i32, [_vp, _i64, _i64, _i64, ctypes.POINTER(ctypes.c_void_p), _i32, _i64, _vp]),
    "dscq_rowquant_tc_noalloc": (_i32, [_vp, _i32, _i64, _i64, _i64, _i32, _i32, _vp, _i32, _f32, _i64, _i64, _vp,
                                        _i64, _vp, _vp, _vp, _vp, _i64, _vp]),
    "dscq_rmsnorm": (_i32, [_vp, _vp, _i64, _i64, _f32, _vp, _vp]),
    "dscq_rope": (_i32, [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _vp]),
    "dscq_silu_mul": (_i32, [_vp, _vp, _i64, _vp, _vp]),
    "dscq_pack_int4": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp]),
    "dscq_unpack_int4": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _vp]),
}

_lib = None
_lock = threading.Lock()


class NativeLibraryMissing(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Loads the native library once (raises NativeLibraryMissing if it was not built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise NativeLibraryMissing(
                        f"{LIB_PATH} is missing; build it with `python -m dscquant_b200.build` "
                        "(the W4A4 path has no CPU or PyTorch fallback)")
                lib = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = lib
    return _lib


def last_error() -> str:
    msg = load().dscq_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    """Maps a C-ABI status to the reference's exception types (TORCH_CHECK -> RuntimeError)."""
    if rc == DSCQ_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == DSCQ_ERR_RANGE:
        raise ValueError(msg)
    raise RuntimeError(msg)
