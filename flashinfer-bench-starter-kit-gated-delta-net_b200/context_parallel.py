"""Context parallelism for few long sequences: one prefill call spread over the ranks
of a process group, each rank holding a contiguous token range of every sequence.

The GDN recurrence is affine in the state: running a token range from initial state
S gives ``S_out = S @ M + C`` per (sequence, v-head), with M [K x K] the range run
from the identity with v taken as 0 and C [V x K] the range run from zero, and the
range's outputs are affine in S too (``o_t = o_t(0) + S @ Phi_t``, Phi the outputs of
the run from the identity).  So:

1. rank 0 runs its ranges from the sequences' initial state (outputs and the state
   leaving its ranges); every other rank meanwhile runs ``kernel_prefill.range_affine``
   on its ranges: their outputs from a zero state, their maps, and (kept on the GPU)
   the homogeneous outputs;
2. one ``all_gather`` of ``[2, N, HV, 128, 128]`` fp32 per rank: rank 0 sends
   ``(0, S_end)``, rank r sends ``(M_r, C_r)`` (the one exchange step of d x d
   matrices per range);
3. rank r > 0 hands the pairs of ranks j < r to ``range_finish``, which folds
   ``S <- S @ M_j + C_j`` from ``S = 0`` on the GPU (rank 0's pair gives ``S_end``) to get
   the state entering its ranges, adds that state's share to its outputs and gives the
   state leaving them (no token runs twice);
4. the last rank's final state is broadcast, so every rank returns the sequences'
   final state.

Both rank 0's prefill and the other ranks' affine pass cut their ranges into segments on
separate SMs; measured on one long 32-head sequence, rank 0's prefill of a range takes
about as long as an affine pass of an equal one, so ``FIRST_RANK_WEIGHT`` is 1.  The
reference has no long-context parallelism (its prefill is token-serial per sequence,
``solution/triton/kernel_prefill.py:88``).

``split_ranges``/``local_inputs`` cut a global varlen batch into rank-local inputs:
every range of a sequence starts on a 64-token chunk boundary.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

CHUNK = 64
FIRST_RANK_WEIGHT = 1.0


def split_ranges(seqlens, world: int, first_weight: float = FIRST_RANK_WEIGHT) -> list[list[tuple[int, int]]]:
    """Per rank, per sequence, the token range ``[lo, hi)`` (sequence-relative) it
    holds: a sequence's chunks are split into ``world`` contiguous runs in proportion
    ``first_weight : 1 : .. : 1`` (rounded down to whole chunks); the last run also
    takes the final partial chunk."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if first_weight <= 0:
        raise ValueError("first_weight must be > 0")
    total = first_weight + (world - 1)
    cum = [0.0] + [(first_weight + r - 1) / total for r in range(1, world)]
    out = [[] for _ in range(world)]
    for L in seqlens:
        L = int(L)
        nch = (L + CHUNK - 1) // CHUNK
        bounds = [min(L, int(cum[r] * nch + 1e-9) * CHUNK) for r in range(world)] + [L]
        for r in range(world):
            out[r].append((bounds[r], bounds[r + 1]))
    return out


def local_inputs(inp: dict, world: int, rank: int, first_weight: float = FIRST_RANK_WEIGHT) -> dict:
    """Rank ``rank``'s slice of a global prefill input dict (keys of ``kernel_prefill.run``):
    its token ranges of every sequence, concatenated, with rank-local ``cu_seqlens``.
    ``state`` is kept on every rank (only rank 0 reads it)."""
    cu = inp["cu_seqlens"].cpu().tolist()
    lens = [cu[i + 1] - cu[i] for i in range(len(cu) - 1)]
    ranges = split_ranges(lens, world, first_weight)[rank]
    parts = [torch.arange(cu[i] + lo, cu[i] + hi, dtype=torch.long) for i, (lo, hi) in enumerate(ranges)]
    idx = torch.cat(parts) if parts else torch.zeros(0, dtype=torch.long)
    local_cu = [0]
    for lo, hi in ranges:
        local_cu.append(local_cu[-1] + hi - lo)
    idx = idx.to(inp["q"].device)
    out = dict(inp)
    for key in ("q", "k", "v", "a", "b"):
        out[key] = inp[key].index_select(0, idx).contiguous()
    out["cu_seqlens"] = torch.tensor(local_cu, dtype=inp["cu_seqlens"].dtype, device=inp["cu_seqlens"].device)
    return out


@dataclass
class Ops:
    """The per-rank computations (the CUDA kernels by default; tests substitute a CPU
    implementation to exercise the exchange on gloo ranks)."""
    prefill: Callable  # (q,k,v,state,A_log,a,dt_bias,b,cu_seqlens,scale) -> (out, final_state)
    affine: Callable  # (q,k,v,A_log,a,dt_bias,b,cu_seqlens,scale) -> (handle, M, C)
    finish: Callable  # (handle, prev [R, 2, N, HV, K, K]: the preceding ranges' (M, C)) -> (out, final_state)


def cuda_ops() -> Ops:
    from . import kernel_prefill

    def affine(q, k, v, A_log, a, dt_bias, b, cu_seqlens, scale):
        h = kernel_prefill.range_affine(q, k, v, A_log, a, dt_bias, b, cu_seqlens, scale)
        return h, h.map_m, h.map_c

    def finish(handle, prev):
        return kernel_prefill.range_finish(handle, prev_maps=prev)

    return Ops(prefill=kernel_prefill.run, affine=affine, finish=finish)


def prefill_context_parallel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, *, group=None,
                             ops: Ops | None = None):
    """One context-parallel prefill step on this rank (inputs as ``kernel_prefill.run``,
    holding this rank's token ranges, e.g. from ``local_inputs``; ``state`` is read on
    rank 0 only and may be None for a zero initial state).  Every rank of ``group``
    calls it with the same sequence count.  Returns ``(output of the local tokens,
    final state of every sequence)``; the final state is the same on every rank."""
    ops = ops or cuda_ops()
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    N = cu_seqlens.shape[0] - 1
    HV, D = v.shape[1], v.shape[2]
    dev = q.device
    if rank == 0:
        out, s_end = ops.prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)
        pair = torch.stack([torch.zeros_like(s_end), s_end])
    else:
        handle, m, c = ops.affine(q, k, v, A_log, a, dt_bias, b, cu_seqlens, scale)
        pair = torch.stack([m, c])
    pairs = torch.empty(world, 2, N, HV, D, D, dtype=torch.float32, device=dev)
    dist.all_gather(list(pairs.unbind(0)), pair.contiguous(), group=group)  # into views of one tensor
    if rank > 0:
        out, s_end = ops.finish(handle, pairs[:rank])
    final = s_end.contiguous() if rank == world - 1 else torch.empty(N, HV, D, D, dtype=torch.float32, device=dev)
    src = dist.get_global_rank(group, world - 1) if group is not None else world - 1
    dist.broadcast(final, src=src, group=group)
    return out, final
