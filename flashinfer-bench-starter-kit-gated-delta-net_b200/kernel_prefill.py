"""GDN varlen prefill operator — drop-in for ``solution/triton/kernel_prefill.py::run``.

``run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale) -> (output, new_state)``
keeps the reference entry point's signature, shapes, dtypes, k-last state
layout and value-returning style (``kernel_prefill.py:234``):

  q, k       bf16 [T, HQ, 128]       v      bf16 [T, HV, 128]
  state      fp32 [N, HV, 128, 128] or None (zeros)
  A_log      fp32 [HV]               dt_bias fp32 [HV]
  a, b       bf16 [T, HV]            cu_seqlens int32/int64 [N + 1] (on the device)
  scale      float, None or 0 -> 1/sqrt(128)
  output     bf16 [T, HV, 128]       new_state fp32 [N, HV, 128, 128] (new buffer)

An empty sequence passes its initial state through, as the reference kernel
does (``kernel_prefill.py:65-73``).  ``run_dps`` is the destination-passing
form.  The work runs in sm_100a kernels through the C ABI ``gdn_prefill`` on
the current CUDA stream (no host synchronisation, no CPU compute).
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

# Workspace buffers cached per (device, stream) so repeated calls do not allocate.
_workspaces: dict = {}


def workspace_size(num_seqs: int, total_tokens: int, num_qk_heads: int, num_v_heads: int,
                   head_dim: int = 128, use_qk_l2norm: bool = False, segments: int = 0) -> int:
    flags = (_lib.GDN_FLAG_QK_L2NORM if use_qk_l2norm else 0) | _lib.GDN_PREFILL_SEGMENTS(segments)
    return int(_lib.library().gdn_prefill_workspace_size(num_seqs, total_tokens, num_qk_heads,
                                                         num_v_heads, head_dim, flags))


def _workspace(device, nbytes: int):
    if nbytes == 0:
        return None
    key = (device, torch.cuda.current_stream(device).cuda_stream)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def run_dps(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state, *,
            use_qk_l2norm: bool = False, serial: bool = False, workspace=None, no_alloc: bool = False,
            segments: int = 0):
    """Destination-passing prefill: writes ``output`` [T,HV,128] bf16 and
    ``new_state`` [N,HV,128,128] fp32 (which may be ``state`` itself).

    The chunked tensor-core kernel runs whenever q/k rows and strides are 16-byte
    aligned (``use_qk_l2norm`` included: the normalisation factors are folded into
    its per-token gate factors); otherwise (or with ``serial=True``, a
    cross-checking switch) the token-serial CUDA kernel runs.
    ``no_alloc=True`` calls ``gdn_prefill_noalloc`` (the library's static scratch
    instead of a workspace buffer; problems larger than it are rejected).
    ``segments`` splits each sequence's chunks into that many ranges run on
    separate SMs (context parallelism; 0 = the library decides, 1 = never)."""
    if not 0 <= int(segments) <= 15:
        raise ValueError(f"segments must be in [0, 15], got {segments}")
    T, HQ, D = q.shape
    HV = v.shape[1]
    N = cu_seqlens.shape[0] - 1
    check_cuda(q, k, v, A_log, a, dt_bias, b, output, new_state, state=state)
    if cu_seqlens.device != q.device:
        raise ValueError("cu_seqlens must be on the same device as q")
    if cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"cu_seqlens must be int32 or int64, got {cu_seqlens.dtype}")
    if scale is None or scale == 0.0:
        scale = 1.0 / math.sqrt(D)
    q, k, v = inner_contig(q), inner_contig(k), inner_contig(v)
    a, b = inner_contig(a), inner_contig(b)
    A_log, dt_bias, cu = A_log.contiguous(), dt_bias.contiguous(), cu_seqlens.contiguous()
    if state is not None and not state.is_contiguous() and state is not new_state:
        state = state.contiguous()
    flags = (_lib.GDN_FLAG_QK_L2NORM if use_qk_l2norm else 0) | (_lib.GDN_FLAG_PREFILL_SERIAL if serial else 0)
    flags |= _lib.GDN_PREFILL_SEGMENTS(segments)
    lib = _lib.library()
    if no_alloc:
        rc = lib.gdn_prefill_noalloc(ptr(q), *seq_head_strides(q, 0, 1), ptr(k), *seq_head_strides(k, 0, 1),
                                     ptr(v), *seq_head_strides(v, 0, 1),
                                     ptr(state), *(seq_head_strides(state, 0, 1) if state is not None else (0, 0)),
                                     ptr(A_log), ptr(a), a.stride(0), ptr(dt_bias), ptr(b), b.stride(0),
                                     ptr(cu), int(cu.dtype == torch.int64),
                                     float(scale),
                                     ptr(output), *seq_head_strides(output, 0, 1),
                                     ptr(new_state), *seq_head_strides(new_state, 0, 1),
                                     N, T, HQ, HV, D, flags, stream_handle(q.device))
        _lib.check(rc)
        return output, new_state
    need = int(lib.gdn_prefill_workspace_size(N, T, HQ, HV, D, flags))
    if workspace is None:
        workspace = _workspace(q.device, need)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = lib.gdn_prefill(ptr(q), *seq_head_strides(q, 0, 1), ptr(k), *seq_head_strides(k, 0, 1),
                         ptr(v), *seq_head_strides(v, 0, 1),
                         ptr(state), *(seq_head_strides(state, 0, 1) if state is not None else (0, 0)),
                         ptr(A_log), ptr(a), a.stride(0), ptr(dt_bias), ptr(b), b.stride(0),
                         ptr(cu), int(cu.dtype == torch.int64),
                         float(scale),
                         ptr(output), *seq_head_strides(output, 0, 1),
                         ptr(new_state), *seq_head_strides(new_state, 0, 1),
                         N, T, HQ, HV, D, ptr(workspace), ws_bytes, flags, stream_handle(q.device))
    _lib.check(rc)
    return output, new_state


def run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, *, use_qk_l2norm: bool = False,
        serial: bool = False, segments: int = 0):
    """Value-returning prefill (the reference's ``run``): returns
    ``(output [T,HV,128] bf16, new_state [N,HV,128,128] fp32)``."""
    T, _, D = q.shape
    HV = v.shape[1]
    N = cu_seqlens.shape[0] - 1
    output = torch.empty(T, HV, D, dtype=torch.bfloat16, device=q.device)
    new_state = torch.empty(N, HV, D, D, dtype=torch.float32, device=q.device)
    return run_dps(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
                   use_qk_l2norm=use_qk_l2norm, serial=serial, segments=segments)


def state_map(q, k, v, A_log, a, dt_bias, b, cu_seqlens, map_m=None, map_c=None, *, workspace=None,
              segments: int = 0):
    """Affine state map of each sequence's token range (C ABI ``gdn_prefill_state_map``):
    running the range from any initial state S gives ``S_out = S @ M + C`` per
    (sequence, v-head), with ``M`` [N,HV,128,128] the range run from the identity with
    v taken as 0 and ``C`` [N,HV,128,128] the range run from zero.  ``segments`` cuts
    each range into that many pieces whose maps are computed on separate SMs and
    multiplied together (0 = the library decides, 1 = one chain per map).  No
    counterpart in the reference; context parallelism composes these maps across ranks."""
    if not 0 <= int(segments) <= 15:
        raise ValueError(f"segments must be in [0, 15], got {segments}")
    T, HQ, D = q.shape
    HV = v.shape[1]
    N = cu_seqlens.shape[0] - 1
    check_cuda(q, k, v, A_log, a, dt_bias, b)
    if cu_seqlens.device != q.device:
        raise ValueError("cu_seqlens must be on the same device as q")
    if cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"cu_seqlens must be int32 or int64, got {cu_seqlens.dtype}")
    if map_m is None:
        map_m = torch.empty(N, HV, D, D, dtype=torch.float32, device=q.device)
    if map_c is None:
        map_c = torch.empty(N, HV, D, D, dtype=torch.float32, device=q.device)
    check_cuda(q, k, v, A_log, a, dt_bias, b, new_state=map_m, state=map_c)
    q, k, v = inner_contig(q), inner_contig(k), inner_contig(v)
    a, b = inner_contig(a), inner_contig(b)
    A_log, dt_bias, cu = A_log.contiguous(), dt_bias.contiguous(), cu_seqlens.contiguous()
    lib = _lib.library()
    flags = _lib.GDN_PREFILL_SEGMENTS(segments)
    need = int(lib.gdn_prefill_workspace_size(N, T, HQ, HV, D, _lib.GDN_FLAG_STATE_MAP | flags))
    if workspace is None:
        workspace = _workspace(q.device, need)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = lib.gdn_prefill_state_map(ptr(q), *seq_head_strides(q, 0, 1), ptr(k), *seq_head_strides(k, 0, 1),
                                   ptr(v), *seq_head_strides(v, 0, 1),
                                   ptr(A_log), ptr(a), a.stride(0), ptr(dt_bias), ptr(b), b.stride(0),
                                   ptr(cu), int(cu.dtype == torch.int64),
                                   ptr(map_m), *seq_head_strides(map_m, 0, 1),
                                   ptr(map_c), *seq_head_strides(map_c, 0, 1),
                                   N, T, HQ, HV, D, ptr(workspace), ws_bytes, flags, stream_handle(q.device))
    _lib.check(rc)
    return map_m, map_c


class RangeHandle:
    """What ``range_affine`` leaves for ``range_finish``: the range's outputs from a zero
    initial state (``out``, completed in place by ``range_finish``), its map
    (``map_m``, ``map_c``) and the workspace holding its segments' maps and homogeneous
    outputs (owned by the handle)."""

    def __init__(self, out, map_m, map_c, workspace, cu, sizes, flags):
        self.out, self.map_m, self.map_c, self.workspace = out, map_m, map_c, workspace
        self.cu, self.sizes, self.flags = cu, sizes, flags


def range_affine(q, k, v, A_log, a, dt_bias, b, cu_seqlens, scale, *, segments: int = 0) -> RangeHandle:
    """First half of the prefill of a later token range of each sequence (context
    parallelism across GPUs; C ABI ``gdn_prefill_range_affine``): the range's outputs from
    a zero initial state and its affine map ``S_out = S_in @ M + C``, before ``S_in`` is
    known.  ``range_finish`` completes the outputs and gives ``S_out`` once it is.  No
    token runs twice.  ``segments`` = map-pair segments per range run on separate SMs
    (0 = the library decides).  No counterpart in the reference."""
    if not 0 <= int(segments) <= 15:
        raise ValueError(f"segments must be in [0, 15], got {segments}")
    T, HQ, D = q.shape
    HV = v.shape[1]
    N = cu_seqlens.shape[0] - 1
    check_cuda(q, k, v, A_log, a, dt_bias, b)
    if cu_seqlens.device != q.device:
        raise ValueError("cu_seqlens must be on the same device as q")
    if cu_seqlens.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"cu_seqlens must be int32 or int64, got {cu_seqlens.dtype}")
    if scale is None or scale == 0.0:
        scale = 1.0 / math.sqrt(D)
    q, k, v = inner_contig(q), inner_contig(k), inner_contig(v)
    a, b = inner_contig(a), inner_contig(b)
    A_log, dt_bias, cu = A_log.contiguous(), dt_bias.contiguous(), cu_seqlens.contiguous()
    out = torch.empty(T, HV, D, dtype=torch.bfloat16, device=q.device)
    map_m = torch.empty(N, HV, D, D, dtype=torch.float32, device=q.device)
    map_c = torch.empty(N, HV, D, D, dtype=torch.float32, device=q.device)
    lib = _lib.library()
    flags = _lib.GDN_FLAG_RANGE_AFFINE | _lib.GDN_PREFILL_SEGMENTS(segments)
    need = int(lib.gdn_prefill_workspace_size(N, T, HQ, HV, D, flags))
    workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    rc = lib.gdn_prefill_range_affine(ptr(q), *seq_head_strides(q, 0, 1), ptr(k), *seq_head_strides(k, 0, 1),
                                      ptr(v), *seq_head_strides(v, 0, 1),
                                      ptr(A_log), ptr(a), a.stride(0), ptr(dt_bias), ptr(b), b.stride(0),
                                      ptr(cu), int(cu.dtype == torch.int64), float(scale),
                                      ptr(out), *seq_head_strides(out, 0, 1),
                                      ptr(map_m), *seq_head_strides(map_m, 0, 1),
                                      ptr(map_c), *seq_head_strides(map_c, 0, 1),
                                      N, T, HQ, HV, D, ptr(workspace), workspace.numel(), flags,
                                      stream_handle(q.device))
    _lib.check(rc)
    return RangeHandle(out, map_m, map_c, workspace, cu, (N, T, HQ, HV, D), flags)


def range_finish(handle: RangeHandle, state_in=None, new_state=None, *, prev_maps=None):
    """Second half (C ABI ``gdn_prefill_range_finish``): given the state entering the range,
    completes ``handle.out`` in place and returns ``(out, S_out)``.  The state is
    ``state_in`` [N,HV,128,128] fp32 (None = zero) or, with ``prev_maps``
    [R,2,N,HV,128,128] fp32 (the (M, C) maps of the R preceding ranges; the first may be
    (0, its final state)), their fold ``S = 0; S = S @ M_j + C_j``, done on the GPU."""
    N, T, HQ, HV, D = handle.sizes
    dev = handle.out.device
    if new_state is None:
        new_state = torch.empty(N, HV, D, D, dtype=torch.float32, device=dev)
    for name, x in (("state_in", state_in), ("new_state", new_state)):
        if x is not None and (x.device != dev or x.dtype != torch.float32 or tuple(x.shape) != (N, HV, D, D)):
            raise ValueError(f"{name} must be a float32 [{N}, {HV}, {D}, {D}] tensor on {dev}")
    count = 0
    if prev_maps is not None:
        if state_in is not None:
            raise ValueError("give either state_in or prev_maps, not both")
        if (prev_maps.device != dev or prev_maps.dtype != torch.float32 or prev_maps.dim() != 6
                or tuple(prev_maps.shape[1:]) != (2, N, HV, D, D)):
            raise ValueError(f"prev_maps must be a float32 [R, 2, {N}, {HV}, {D}, {D}] tensor on {dev}")
        prev_maps = prev_maps.contiguous()
        count = prev_maps.shape[0]
    if state_in is not None and not state_in.is_contiguous() and state_in is not new_state:
        state_in = state_in.contiguous()
    lib = _lib.library()
    rc = lib.gdn_prefill_range_finish(ptr(handle.cu), int(handle.cu.dtype == torch.int64),
                                      ptr(state_in), *(seq_head_strides(state_in, 0, 1) if state_in is not None
                                                       else (0, 0)),
                                      ptr(prev_maps) if count else None, count,
                                      ptr(handle.out), *seq_head_strides(handle.out, 0, 1),
                                      ptr(new_state), *seq_head_strides(new_state, 0, 1),
                                      N, T, HQ, HV, D, ptr(handle.workspace), handle.workspace.numel(),
                                      handle.flags, stream_handle(dev))
    _lib.check(rc)
    return handle.out, new_state
