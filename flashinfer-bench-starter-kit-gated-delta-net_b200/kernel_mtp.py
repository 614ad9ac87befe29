"""GDN multi-token decode against a state pool (the serving / MTP form).

``run(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale,
intermediate_states_buffer=None) -> (output, final_state)`` keeps the argument
list, shapes and semantics of the definition-level reference
``_gdn_mtp_reference`` (flashinfer 0.6.11.post2,
``flashinfer/trace/templates/gdn.py``; the starter kit's own decode handles one
token against a dense state batch):

  q, k            bf16 [B, T, HQ, 128]       v       bf16 [B, T, HV, 128]
  initial_state   fp32 [P, HV, 128, 128]     initial_state_indices int32/int64 [B]
  A_log, dt_bias  fp32 [HV]                  a, b    bf16 [B, T, HV]
  scale           float, None or 0 -> 1/sqrt(128)
  output          bf16 [B, T, HV, 128]       final_state fp32 [P, HV, 128, 128]
  intermediate_states_buffer  optional fp32 [P, T, HV, 128, 128]: the state
                  after every token, written to the sequence's slot

Sequence b runs T decode steps from ``initial_state[initial_state_indices[b]]``;
``final_state`` is a copy of the pool with those slots replaced (as the
reference returns).  ``run_dps`` writes into a caller-provided ``final_state``
that may be ``initial_state`` itself (in-place serving update, no pool copy).
Indices must be distinct; a negative index skips its sequence (zero outputs,
slot untouched) — the serving convention for padded batch entries, where the
reference would index from the end of the pool.  The state crosses HBM once per
call whatever T is (one launch of an sm_100a kernel through the C ABI
``gdn_decode_pooled``).
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
    from gdn_b200._tensors import check_cuda, ptr, stream_handle, inner_contig
else:
    from . import _lib
    from ._tensors import check_cuda, ptr, stream_handle, inner_contig


def _strides3(t):
    return t.stride(0), t.stride(1), t.stride(2)


def _pool_strides(t):
    if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1]:
        raise ValueError("state pools need row-major [V, K] blocks (k-last layout)")
    return t.stride(0), t.stride(1)


def run_dps(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale, output, final_state,
            intermediate_states_buffer=None, *, use_qk_l2norm: bool = False):
    """Destination-passing form: writes ``output`` [B,T,HV,128] and the slots of
    ``final_state`` (which may be ``initial_state``) named by the indices."""
    B, T, HQ, D = q.shape
    HV = v.shape[2]
    P = initial_state.shape[0]
    check_cuda(q, k, v, A_log, a, dt_bias, b, output, final_state, state=initial_state)
    idx = initial_state_indices
    if idx.device != q.device:
        raise ValueError("initial_state_indices must be on the same device as q")
    if idx.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"initial_state_indices must be int32 or int64, got {idx.dtype}")
    if tuple(idx.shape) != (B,):
        raise ValueError(f"initial_state_indices must have shape [{B}], got {tuple(idx.shape)}")
    inter = intermediate_states_buffer
    if inter is not None:
        if inter.dtype != torch.float32 or inter.device != q.device or tuple(inter.shape) != (P, T, HV, D, D):
            raise ValueError(f"intermediate_states_buffer must be float32 [{P}, {T}, {HV}, {D}, {D}] on {q.device}")
        if inter.stride(-1) != 1 or inter.stride(-2) != D:
            raise ValueError("intermediate_states_buffer needs row-major [V, K] blocks")
    if scale is None or scale == 0.0:
        scale = 1.0 / math.sqrt(D)
    q, k, v = inner_contig(q), inner_contig(k), inner_contig(v)
    a, b = inner_contig(a), inner_contig(b)
    A_log, dt_bias, idx = A_log.contiguous(), dt_bias.contiguous(), idx.contiguous()
    lib = _lib.library()
    rc = lib.gdn_decode_pooled(ptr(q), *_strides3(q), ptr(k), *_strides3(k), ptr(v), *_strides3(v),
                               ptr(initial_state), *_pool_strides(initial_state),
                               ptr(idx), int(idx.dtype == torch.int64),
                               ptr(A_log), ptr(a), a.stride(0), a.stride(1), ptr(dt_bias), ptr(b), b.stride(0),
                               b.stride(1), float(scale),
                               ptr(output), *_strides3(output),
                               ptr(final_state), *_pool_strides(final_state),
                               ptr(inter), *(_strides3(inter) if inter is not None else (0, 0, 0)),
                               B, T, P, HQ, HV, D, _lib.GDN_FLAG_QK_L2NORM if use_qk_l2norm else 0,
                               stream_handle(q.device))
    _lib.check(rc)
    return output, final_state


def run(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale,
        intermediate_states_buffer=None, *, use_qk_l2norm: bool = False):
    """Value-returning form (``_gdn_mtp_reference``'s): returns ``(output, final_state)``
    with ``final_state`` a new pool (a copy of ``initial_state`` with the indexed
    slots advanced by T tokens)."""
    B, T, _, D = q.shape
    HV = v.shape[2]
    output = torch.empty(B, T, HV, D, dtype=torch.bfloat16, device=q.device)
    final_state = initial_state.clone()
    return run_dps(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale, output,
                   final_state, intermediate_states_buffer, use_qk_l2norm=use_qk_l2norm)
