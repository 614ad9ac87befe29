"""Seeded inputs shared by the golden generator and the tests.

The 16/32-head fixtures do not store their inputs (they would be several MB):
the tests regenerate them here from the seed with torch's CPU generator and
check them against the SHA-256 digest stored in the fixture, so an input drift
fails loudly instead of comparing against the wrong outputs.
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def make_inputs(shape_q, shape_v, shape_g, state_shape, seed):
    """q, k unit rows (bf16), v, a, b ~ N(0, 1) (bf16), A_log ~ U(0, 1.5), dt_bias ~ U(-1, 1),
    state ~ N(0, 0.05) rounded to bf16-representable fp32 values."""
    gen = torch.Generator()
    gen.manual_seed(seed)

    def unit(shape):
        x = torch.randn(*shape, generator=gen)
        return (x / x.norm(dim=-1, keepdim=True)).bfloat16()

    q, k = unit(shape_q), unit(shape_q)
    v = torch.randn(*shape_v, generator=gen).bfloat16()
    a = torch.randn(*shape_g, generator=gen).bfloat16()
    b = torch.randn(*shape_g, generator=gen).bfloat16()
    HV = shape_v[-2]
    A_log = torch.rand(HV, generator=gen) * 1.5
    dt_bias = torch.rand(HV, generator=gen) * 2 - 1
    state = (torch.randn(*state_shape, generator=gen) * 0.05).bfloat16().float()
    return q, k, v, a, b, A_log, dt_bias, state


def digest(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


# The 16/32-head cases (BASELINE.json's head counts; GVA ratio 2).  States are stored
# for the v-heads below only (pairs sharing a q/k head at both ends of the head range
# and in the middle); the outputs cover every head.
HQ16, HV32 = 16, 32
STORED_HEADS = [0, 1, 14, 15, 16, 17, 30, 31]


def decode_qk16v32_inputs(seed: int = 13, B: int = 2):
    return make_inputs((B, 1, HQ16, 128), (B, 1, HV32, 128), (B, 1, HV32), (B, HV32, 128, 128), seed)


def prefill_qk16v32_inputs(lens, seed: int = 22):
    T, N = sum(lens), len(lens)
    q, k, v, a, b, A_log, dt_bias, state = make_inputs(
        (T, HQ16, 128), (T, HV32, 128), (T, HV32), (N, HV32, 128, 128), seed)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    return q, k, v, a, b, A_log, dt_bias, state, cu
