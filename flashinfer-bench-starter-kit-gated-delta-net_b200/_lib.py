"""ctypes binding of ``libgdn_b200.so`` (the C ABI of ``include/gdn_b200.h``).

The library is loaded lazily on first use.  If it is missing or fails to load
every operator raises ``RuntimeError``; there is no fallback implementation.
Set ``GDN_B200_LIB`` to load a library from another path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
_DEFAULT = _HERE / "libgdn_b200.so"

GDN_OK = 0
GDN_ERR_INVALID_ARGUMENT = 1
GDN_ERR_UNSUPPORTED = 2
GDN_ERR_CUDA = 3
GDN_ERR_WORKSPACE = 4
GDN_FLAG_QK_L2NORM = 0x1
GDN_FLAG_PREFILL_SERIAL = 0x2
GDN_FLAG_STATE_MAP = 0x4
GDN_FLAG_RANGE_AFFINE = 0x8
GDN_FLAG_SELFTEST_WAIT_TIMEOUT = 0x80000000


def GDN_PREFILL_SEGMENTS(n: int) -> int:
    """Flag bits requesting n context-parallel segments per sequence (0 = automatic, 1 = none)."""
    return (int(n) & 15) << 8

GDN_DEVERR_WAIT_TIMEOUT = 0x1
GDN_DEVERR_BAD_SEQLENS = 0x2
GDN_DEVERR_BAD_INDEX = 0x4
GDN_PREFILL_NOALLOC_SCRATCH_BYTES = 64 << 20

# Every symbol the header declares, with its ctypes signature.
_P, _I64, _I32, _U32, _F, _SZ = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_uint32,
                                  ctypes.c_float, ctypes.c_size_t)
SIGNATURES = {
    "gdn_version": ([], ctypes.c_int),
    "gdn_last_error": ([], ctypes.c_char_p),
    "gdn_device_error": ([ctypes.POINTER(ctypes.c_uint32), ctypes.c_int], ctypes.c_int),
    "gdn_decode": ([_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,   # q, k, v
                    _P, _I64, _I64,                                    # state
                    _P, _P, _I64, _P, _P, _I64,                        # A_log, a, dt_bias, b
                    _F,                                                # scale
                    _P, _I64, _I64, _P, _I64, _I64,                    # out, new_state
                    _I32, _I32, _I32, _I32, _U32, _P], ctypes.c_int),
    "gdn_prefill": ([_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,  # q, k, v
                     _P, _I64, _I64,                                   # state
                     _P, _P, _I64, _P, _P, _I64,                       # A_log, a, dt_bias, b
                     _P, _I32,                                         # cu_seqlens
                     _F,                                               # scale
                     _P, _I64, _I64, _P, _I64, _I64,                   # out, new_state
                     _I32, _I64, _I32, _I32, _I32,                     # N, T, HQ, HV, D
                     _P, _SZ, _U32, _P], ctypes.c_int),
    "gdn_prefill_workspace_size": ([_I32, _I64, _I32, _I32, _I32, _U32], ctypes.c_size_t),
    "gdn_decode_pooled": ([_P, _I64, _I64, _I64, _P, _I64, _I64, _I64,   # q, k
                           _P, _I64, _I64, _I64,                         # v
                           _P, _I64, _I64, _P, _I32,                     # pool, indices
                           _P, _P, _I64, _I64, _P, _P, _I64, _I64,       # A_log, a, dt_bias, b
                           _F,                                           # scale
                           _P, _I64, _I64, _I64,                         # out
                           _P, _I64, _I64,                               # new_pool
                           _P, _I64, _I64, _I64,                         # intermediate
                           _I32, _I32, _I32, _I32, _I32, _I32, _U32, _P], ctypes.c_int),
    "gdn_prefill_noalloc": ([_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,  # q, k, v
                             _P, _I64, _I64,                                   # state
                             _P, _P, _I64, _P, _P, _I64,                       # A_log, a, dt_bias, b
                             _P, _I32,                                         # cu_seqlens
                             _F,                                               # scale
                             _P, _I64, _I64, _P, _I64, _I64,                   # out, new_state
                             _I32, _I64, _I32, _I32, _I32,                     # N, T, HQ, HV, D
                             _U32, _P], ctypes.c_int),
    "gdn_prefill_state_map": ([_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,  # q, k, v
                               _P, _P, _I64, _P, _P, _I64,                       # A_log, a, dt_bias, b
                               _P, _I32,                                         # cu_seqlens
                               _P, _I64, _I64, _P, _I64, _I64,                   # map_m, map_c
                               _I32, _I64, _I32, _I32, _I32,                     # N, T, HQ, HV, D
                               _P, _SZ, _U32, _P], ctypes.c_int),
    "gdn_prefill_range_affine": ([_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,  # q, k, v
                                  _P, _P, _I64, _P, _P, _I64,                       # A_log, a, dt_bias, b
                                  _P, _I32, _F,                                     # cu_seqlens, scale
                                  _P, _I64, _I64,                                   # out
                                  _P, _I64, _I64, _P, _I64, _I64,                   # map_m, map_c
                                  _I32, _I64, _I32, _I32, _I32,                     # N, T, HQ, HV, D
                                  _P, _SZ, _U32, _P], ctypes.c_int),
    "gdn_prefill_range_finish": ([_P, _I32,                                         # cu_seqlens
                                  _P, _I64, _I64,                                   # state (S_in)
                                  _P, _I32,                                         # prev_maps, count
                                  _P, _I64, _I64,                                   # out
                                  _P, _I64, _I64,                                   # new_state
                                  _I32, _I64, _I32, _I32, _I32,                     # N, T, HQ, HV, D
                                  _P, _SZ, _U32, _P], ctypes.c_int),
}

_lib = None


class GDNError(RuntimeError):
    """Raised when a C-ABI call returns a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"gdn_b200 error {code}: {message}")
        self.code = code


def library_path() -> Path:
    return Path(os.environ.get("GDN_B200_LIB", str(_DEFAULT)))


def library():
    """The loaded ``ctypes.CDLL`` (raises ``RuntimeError`` if it is not built)."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.exists():
        raise RuntimeError(
            f"gdn_b200: CUDA library {path} is not built (run build.py or __graft_entry__.build()); "
            "there is no fallback implementation")
    lib = ctypes.CDLL(str(path))
    for name, (argtypes, restype) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != GDN_OK:
        msg = library().gdn_last_error()
        raise GDNError(rc, msg.decode() if msg else "")


def device_error(clear: bool = True) -> int:
    """Device-side error bits (synchronises the current device)."""
    bits = ctypes.c_uint32(0)
    check(library().gdn_device_error(ctypes.byref(bits), int(clear)))
    return bits.value
