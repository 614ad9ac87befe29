"""GDN decode operator — drop-in for ``solution/triton/kernel_decode.py::run``.

``run(q, k, v, state, A_log, a, dt_bias, b, scale) -> (output, new_state)``
keeps the reference entry point's signature, tensor shapes, dtypes, k-last
state layout and value-returning style (``kernel_decode.py:186``,
``config.toml:9`` ``destination_passing_style = false``):

  q, k      bf16  [B, 1, HQ, 128]        v     bf16 [B, 1, HV, 128]
  state     fp32  [B, HV, 128, 128] or None (zeros)
  A_log     fp32  [HV]                   dt_bias fp32 [HV]
  a, b      bf16  [B, 1, HV]             scale   float, None or 0 -> 1/sqrt(128)
  output    bf16  [B, 1, HV, 128]        new_state fp32 [B, HV, 128, 128] (new buffer)

``run_dps`` is the destination-passing form (outputs passed last, in the
definition's output order) and accepts ``new_state is state`` for an in-place
update.  The work is one launch of the fused sm_100a decode kernel through the
C ABI ``gdn_decode`` on the current CUDA stream; nothing here computes on the
CPU.  Loading this file by path (the harness's ``kernel_decode.py::run``
entry-point form) works as well as importing it from the package.
"""
from __future__ import annotations

import math
import sys
from pathlib import Path

import torch

if __package__ in (None, ""):  # loaded by file path: register the package first
    import importlib.util

    _dir = Path(__file__).resolve().parent
    if "gdn_b200" not in sys.modules:
        _spec = importlib.util.spec_from_file_location(
            "gdn_b200", _dir / "__init__.py", submodule_search_locations=[str(_dir)])
        _mod = importlib.util.module_from_spec(_spec)
        sys.modules["gdn_b200"] = _mod
        _spec.loader.exec_module(_mod)
    from gdn_b200 import _lib
    from gdn_b200._tensors import check_cuda, ptr, stream_handle, inner_contig, seq_head_strides
else:
    from . import _lib
    from ._tensors import check_cuda, ptr, stream_handle, inner_contig, seq_head_strides


def _flags(use_qk_l2norm: bool) -> int:
    return _lib.GDN_FLAG_QK_L2NORM if use_qk_l2norm else 0


def run_dps(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state, *,
            use_qk_l2norm: bool = False, extra_flags: int = 0):
    """Destination-passing decode: writes ``output`` [B,1,HV,128] bf16 and
    ``new_state`` [B,HV,128,128] fp32 (which may be ``state`` itself).
    ``extra_flags`` are further C-ABI flag bits (``GDN_FLAG_SELFTEST_WAIT_TIMEOUT``)."""
    B, T1, HQ, D = q.shape
    HV = v.shape[2]
    if T1 != 1:
        raise ValueError(f"decode expects one token per sequence (q.shape[1] == 1), got {T1}")
    check_cuda(q, k, v, A_log, a, dt_bias, b, output, new_state, state=state)
    if scale is None or scale == 0.0:
        scale = 1.0 / math.sqrt(D)
    q, k, v = inner_contig(q), inner_contig(k), inner_contig(v)
    a, b = inner_contig(a, dims=2), inner_contig(b, dims=2)
    A_log, dt_bias = A_log.contiguous(), dt_bias.contiguous()
    if state is not None and not state.is_contiguous() and state is not new_state:
        state = state.contiguous()
    sq = seq_head_strides(q, 0, 2)
    sk = seq_head_strides(k, 0, 2)
    sv = seq_head_strides(v, 0, 2)
    ss = seq_head_strides(state, 0, 1) if state is not None else (0, 0)
    so = seq_head_strides(output, 0, 2)
    sn = seq_head_strides(new_state, 0, 1)
    lib = _lib.library()
    rc = lib.gdn_decode(ptr(q), *sq, ptr(k), *sk, ptr(v), *sv,
                        ptr(state), *ss,
                        ptr(A_log), ptr(a), a.stride(0), ptr(dt_bias), ptr(b), b.stride(0),
                        float(scale),
                        ptr(output), *so, ptr(new_state), *sn,
                        B, HQ, HV, D, _flags(use_qk_l2norm) | int(extra_flags), stream_handle(q.device))
    _lib.check(rc)
    return output, new_state


def run(q, k, v, state, A_log, a, dt_bias, b, scale, *, use_qk_l2norm: bool = False):
    """Value-returning decode (the reference's ``run``): returns
    ``(output [B,1,HV,128] bf16, new_state [B,HV,128,128] fp32)``."""
    B, _, _, D = q.shape
    HV = v.shape[2]
    output = torch.empty(B, 1, HV, D, dtype=torch.bfloat16, device=q.device)
    new_state = torch.empty(B, HV, D, D, dtype=torch.float32, device=q.device)
    return run_dps(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state,
                   use_qk_l2norm=use_qk_l2norm)
