"""Small tensor helpers shared by the operator wrappers (no compute)."""
from __future__ import annotations

import torch

_BF16 = torch.bfloat16
_F32 = torch.float32

# Expected dtype per argument name (the definitions' dtypes).
DTYPES = {"q": _BF16, "k": _BF16, "v": _BF16, "a": _BF16, "b": _BF16, "output": _BF16,
          "A_log": _F32, "dt_bias": _F32, "state": _F32, "new_state": _F32}


def check_cuda(q, k, v, A_log, a, dt_bias, b, output=None, new_state=None, state=None):
    """All tensors on one CUDA device with the definition's dtypes (output, new_state
    and state are checked when given)."""
    named = dict(q=q, k=k, v=v, A_log=A_log, a=a, dt_bias=dt_bias, b=b)
    for name, t in (("output", output), ("new_state", new_state), ("state", state)):
        if t is not None:
            named[name] = t
    dev = q.device
    if dev.type != "cuda":
        raise RuntimeError("gdn_b200 operators run on CUDA tensors only (no CPU implementation)")
    for name, t in named.items():
        if not torch.is_tensor(t):
            raise TypeError(f"{name} must be a tensor")
        if t.device != dev:
            raise ValueError(f"{name} is on {t.device}, expected {dev}")
        if t.dtype != DTYPES[name]:
            raise TypeError(f"{name} must be {DTYPES[name]}, got {t.dtype}")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def inner_contig(t, dims: int = 1):
    """Return ``t`` if its last ``dims`` dimensions are densely packed, else a
    contiguous copy (the reference's wrapper makes the same ``.contiguous()``
    copies, ``kernel_decode.py:127-131``)."""
    expected = 1
    for d in range(t.dim() - 1, t.dim() - 1 - dims, -1):
        if t.shape[d] != 1 and t.stride(d) != expected:
            return t.contiguous()
        expected *= t.shape[d]
    return t


def seq_head_strides(t, d_seq: int, d_head: int):
    """(sequence stride, head stride) in elements; for 4-D states the inner
    [V, K] block must be row-major."""
    if t.dim() == 4 and t.shape[-1] == t.shape[-2] and t.dtype == _F32:
        if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1]:
            raise ValueError("state tensors need row-major [V, K] blocks (k-last layout)")
    return t.stride(d_seq), t.stride(d_head)
