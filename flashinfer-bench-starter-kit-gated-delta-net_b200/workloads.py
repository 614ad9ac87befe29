"""Seeded synthetic GDN workloads with the shapes and value distributions of the
benchmark configurations (decode batches, varlen and long-context prefill).

The reference is measured on the ``flashinfer-ai/mlsys26-contest`` dataset
workloads (``README.md:53-66`` of the reference), which are not available
offline; these generators stand in for them with the same per-token layout:
d = 128, GVA ratio HV / HQ = 2, k-last fp32 state ``[.., HV, V, K]``, bf16
activations.

Distributions (all drawn from one ``torch.Generator`` seeded per workload):
  q, k     bf16, N(0, 1) drawn in fp32, L2-normalised over d, then cast to bf16
  v, a, b  bf16, N(0, 1)
  A_log    fp32, U(0, 1.5)          [HV]
  dt_bias  fp32, U(-1, 1)           [HV]
  state    fp32, N(0, 0.05^2)       (or zeros for the long-context prefill)
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

HEAD_DIM = 128
NUM_QK_HEADS = 16
NUM_V_HEADS = 32
STATE_STD = 0.05


def _normal(gen, shape, device):
    return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32)


def _unit_bf16(gen, shape, device):
    x = _normal(gen, shape, device)
    x = x / x.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    return x.to(torch.bfloat16)


def _gate_params(gen, HV, device):
    A_log = torch.rand(HV, generator=gen, device=device) * 1.5
    dt_bias = torch.rand(HV, generator=gen, device=device) * 2.0 - 1.0
    return A_log.float(), dt_bias.float()


def decode_inputs(batch: int, num_qk_heads: int = NUM_QK_HEADS, num_v_heads: int = NUM_V_HEADS,
                  head_dim: int = HEAD_DIM, seed: int = 0, device="cpu", zero_state: bool = False,
                  state_std: float = STATE_STD) -> dict:
    """Inputs of one decode step, keyed by the reference's argument names
    (``kernel_decode.py:186``: q, k, v, state, A_log, a, dt_bias, b, scale)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    B, HQ, HV, D = batch, num_qk_heads, num_v_heads, head_dim
    q = _unit_bf16(gen, (B, 1, HQ, D), device)
    k = _unit_bf16(gen, (B, 1, HQ, D), device)
    v = _normal(gen, (B, 1, HV, D), device).to(torch.bfloat16)
    a = _normal(gen, (B, 1, HV), device).to(torch.bfloat16)
    b = _normal(gen, (B, 1, HV), device).to(torch.bfloat16)
    A_log, dt_bias = _gate_params(gen, HV, device)
    if zero_state:
        state = torch.zeros(B, HV, D, D, device=device)
    else:
        state = _normal(gen, (B, HV, D, D), device) * state_std
    return dict(q=q, k=k, v=v, state=state, A_log=A_log, a=a, dt_bias=dt_bias, b=b,
                scale=1.0 / math.sqrt(D))


def prefill_inputs(seqlens, num_qk_heads: int = NUM_QK_HEADS, num_v_heads: int = NUM_V_HEADS,
                   head_dim: int = HEAD_DIM, seed: int = 0, device="cpu", zero_state: bool = False,
                   state_std: float = STATE_STD, cu_dtype=torch.int32) -> dict:
    """Inputs of one varlen prefill call, keyed by the reference's argument
    names (``kernel_prefill.py:234``: q, k, v, state, A_log, a, dt_bias, b,
    cu_seqlens, scale)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    lens = [int(x) for x in seqlens]
    N, T = len(lens), sum(lens)
    HQ, HV, D = num_qk_heads, num_v_heads, head_dim
    q = _unit_bf16(gen, (T, HQ, D), device)
    k = _unit_bf16(gen, (T, HQ, D), device)
    v = _normal(gen, (T, HV, D), device).to(torch.bfloat16)
    a = _normal(gen, (T, HV), device).to(torch.bfloat16)
    b = _normal(gen, (T, HV), device).to(torch.bfloat16)
    A_log, dt_bias = _gate_params(gen, HV, device)
    if zero_state:
        state = torch.zeros(N, HV, D, D, device=device)
    else:
        state = _normal(gen, (N, HV, D, D), device) * state_std
    cu = torch.zeros(N + 1, dtype=torch.int64)
    cu[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int64), 0)
    return dict(q=q, k=k, v=v, state=state, A_log=A_log, a=a, dt_bias=dt_bias, b=b,
                cu_seqlens=cu.to(cu_dtype).to(device), scale=1.0 / math.sqrt(D))


def varlen_seqlens(num_seqs: int = 16, lo: int = 128, hi: int = 4096, seed: int = 0):
    """Sequence lengths drawn uniformly from [lo, hi] with a fixed seed."""
    gen = torch.Generator()
    gen.manual_seed(seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (num_seqs,), generator=gen)]


@dataclass(frozen=True)
class Workload:
    """One benchmark configuration (index into the published config list)."""
    name: str
    kind: str          # "decode" | "prefill"
    batch: int = 0     # decode: sequences per step
    seqlens: tuple = ()  # prefill: per-sequence token counts
    zero_state: bool = False

    @property
    def num_tokens(self) -> int:
        return self.batch if self.kind == "decode" else sum(self.seqlens)


def config(index: int) -> Workload:
    """The five published configurations (0: CPU decode B=1, 1: decode B=64,
    2: decode B=1024, 3: varlen prefill 16 x U[128, 4096], 4: 8 x 32768 prefill)."""
    if index == 0:
        return Workload("decode_b1", "decode", batch=1)
    if index == 1:
        return Workload("decode_b64", "decode", batch=64)
    if index == 2:
        return Workload("decode_b1024", "decode", batch=1024)
    if index == 3:
        return Workload("prefill_varlen16", "prefill", seqlens=tuple(varlen_seqlens()))
    if index == 4:
        return Workload("prefill_8x32768", "prefill", seqlens=(32768,) * 8, zero_state=True)
    raise IndexError(index)


# Algorithmic cost model (fixed formulas; used for GB/s and roofline fractions).
def decode_bytes_per_seq(num_qk_heads=NUM_QK_HEADS, num_v_heads=NUM_V_HEADS, d=HEAD_DIM) -> int:
    """State read + write (fp32) plus q, k, v, o (bf16) and a, b (bf16) per sequence step."""
    return (num_v_heads * d * d * 4 * 2 + num_qk_heads * d * 2 * 2 + num_v_heads * d * 2 * 2
            + num_v_heads * 2 * 2)


def mtp_bytes_per_seq(tokens, num_qk_heads=NUM_QK_HEADS, num_v_heads=NUM_V_HEADS, d=HEAD_DIM) -> int:
    """Pooled multi-token decode, one sequence: its state slot read + written once
    (fp32) plus q, k, v, o (bf16) and a, b (bf16) of every token (no intermediate
    states cached)."""
    return (num_v_heads * d * d * 4 * 2
            + tokens * (num_qk_heads * d * 2 * 2 + num_v_heads * d * 2 * 2 + num_v_heads * 2 * 2))


def prefill_flops_per_token(num_v_heads=NUM_V_HEADS, d=HEAD_DIM, chunk=64) -> float:
    """Chunked WY/UT FLOPs per token: HV * (10*C*d + 6*d^2 + (2/3)*C^2)."""
    return num_v_heads * (10 * chunk * d + 6 * d * d + (2.0 / 3.0) * chunk * chunk)


def prefill_bytes(num_tokens, num_seqs, num_qk_heads=NUM_QK_HEADS, num_v_heads=NUM_V_HEADS,
                  d=HEAD_DIM) -> int:
    """q, k, v, o (bf16) and a, b per token, plus initial + final fp32 state per sequence."""
    per_tok = num_qk_heads * d * 2 * 2 + num_v_heads * d * 2 * 2 + num_v_heads * 2 * 2
    return num_tokens * per_tok + num_seqs * num_v_heads * d * d * 4 * 2
