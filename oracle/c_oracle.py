"""ctypes wrapper for the C restatement ``oracle/gdn_oracle.c`` (test infrastructure only)."""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_DIR = Path(__file__).resolve().parent
LIB_PATH = _DIR / "_build" / "libgdn_oracle.so"
_lib = None


def build(force: bool = False) -> Path:
    """Compile ``gdn_oracle.c`` with the committed Makefile."""
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (_DIR / "gdn_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_DIR)], check=True)
    return LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        I = ctypes.c_int
        lib.gdn_oracle_decode.argtypes = [P, P, P, P, P, P, P, P, ctypes.c_float, I, P, P, I, I, I, I, I]
        lib.gdn_oracle_decode.restype = I
        lib.gdn_oracle_prefill.argtypes = [P, P, P, P, P, P, P, P, P, ctypes.c_float, I, P, P, I, I, I, I, I]
        lib.gdn_oracle_prefill.restype = I
        _lib = lib
    return _lib


def _p(x):
    return None if x is None else x.ctypes.data_as(ctypes.c_void_p)


def _c(x, dt):
    return None if x is None else np.ascontiguousarray(x, dtype=dt)


def default_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def decode(q, k, v, state, A_log, a, dt_bias, b, scale=None, use_qk_l2norm=False, nthreads=None):
    """Same contract as ``gdn_oracle.decode`` (bf16 as uint16 bits)."""
    lib = _load()
    B, _, HQ, D = q.shape
    HV = v.shape[2]
    q, k, v = _c(q, np.uint16), _c(k, np.uint16), _c(v, np.uint16)
    a, b = _c(a, np.uint16), _c(b, np.uint16)
    state = _c(state, np.float32)
    A_log, dt_bias = _c(A_log, np.float32), _c(dt_bias, np.float32)
    out = np.empty((B, 1, HV, D), np.uint16)
    new_state = np.empty((B, HV, D, D), np.float32)
    rc = lib.gdn_oracle_decode(_p(q), _p(k), _p(v), _p(state), _p(A_log), _p(a), _p(dt_bias), _p(b),
                               0.0 if scale is None else float(scale), int(use_qk_l2norm), _p(out),
                               _p(new_state), B, HQ, HV, D, nthreads or default_threads())
    if rc != 0:
        raise ValueError(f"gdn_oracle_decode failed ({rc})")
    return out, new_state


def prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None, use_qk_l2norm=False,
            nthreads=None):
    """Same contract as ``gdn_oracle.prefill`` (bf16 as uint16 bits)."""
    lib = _load()
    T, HQ, D = q.shape
    HV = v.shape[1]
    cu = _c(cu_seqlens, np.int64)
    N = cu.shape[0] - 1
    q, k, v = _c(q, np.uint16), _c(k, np.uint16), _c(v, np.uint16)
    a, b = _c(a, np.uint16), _c(b, np.uint16)
    state = _c(state, np.float32)
    A_log, dt_bias = _c(A_log, np.float32), _c(dt_bias, np.float32)
    out = np.zeros((T, HV, D), np.uint16)
    new_state = np.empty((N, HV, D, D), np.float32)
    rc = lib.gdn_oracle_prefill(_p(q), _p(k), _p(v), _p(state), _p(A_log), _p(a), _p(dt_bias), _p(b),
                                _p(cu), 0.0 if scale is None else float(scale), int(use_qk_l2norm),
                                _p(out), _p(new_state), N, HQ, HV, D, nthreads or default_threads())
    if rc != 0:
        raise ValueError(f"gdn_oracle_prefill failed ({rc})")
    return out, new_state
