"""Multi-GPU work split for GDN decode and prefill (one process per GPU).

Every (sequence, v-head) state evolves independently, so both operators shard
without any exchange on the hot path: a rank owns a slice of sequences (and,
for few long prefill sequences, a slice of v-head pairs) together with their
states.  Nothing here launches a collective; ``gather_to_rank0`` is the only
optional NCCL step, for callers that need every output on one rank.

v-heads are split in pairs (2j, 2j+1 share q/k head j when HV/HQ = 2), so a
head slice never splits the q/k head it reads.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass, field


def batch_slice(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced [start, end) slice of a decode batch for ``rank``."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass
class PrefillShard:
    """Work of one rank: sequences (indices into the call's cu_seqlens) and the
    v-head range [head_lo, head_hi) it computes for each of them."""
    rank: int
    seqs: list = field(default_factory=list)
    head_lo: int = 0
    head_hi: int = 0
    tokens: int = 0  # tokens x (head share) of assigned work, for balance checks

    @property
    def units(self) -> float:
        return self.tokens


def plan_prefill(seqlens, num_v_heads: int, world: int, head_group: int = 2) -> list[PrefillShard]:
    """Split a varlen prefill over ``world`` ranks.

    * ``len(seqlens) >= world``: whole sequences, longest-first greedy onto the
      least-loaded rank (LPT), every rank computes all heads.
    * fewer sequences than ranks: every rank takes all sequences and a
      contiguous block of v-head groups (``world`` must divide the number of
      head groups).
    """
    lens = [int(x) for x in seqlens]
    if world <= 0:
        raise ValueError("world must be positive")
    if world == 1 or len(lens) >= world:
        shards = [PrefillShard(r, head_lo=0, head_hi=num_v_heads) for r in range(world)]
        heap = [(0, r) for r in range(world)]
        for i in sorted(range(len(lens)), key=lambda i: (-lens[i], i)):
            load, r = heapq.heappop(heap)
            shards[r].seqs.append(i)
            shards[r].tokens += lens[i]
            heapq.heappush(heap, (load + lens[i], r))
        for s in shards:
            s.seqs.sort()
        return shards
    groups = num_v_heads // head_group
    if num_v_heads % head_group or groups % world:
        raise ValueError(f"{num_v_heads} v-heads in groups of {head_group} do not split over {world} ranks")
    per = groups // world
    total = sum(lens)
    return [PrefillShard(r, seqs=list(range(len(lens))), head_lo=r * per * head_group,
                         head_hi=(r + 1) * per * head_group, tokens=total * per * head_group // num_v_heads)
            for r in range(world)]


def prefill_shard_calls(shard: PrefillShard, seqlens, q, k, v, state, A_log, a, dt_bias, b, output, new_state,
                        cu_dtype=None):
    """The prefill calls of one rank's share, as keyword arguments for
    ``kernel_prefill.run_dps``: one call per contiguous run of the shard's sequences,
    every tensor a view of the full call's tensors restricted to the run's tokens and
    the shard's v-head range (q/k to the q/k heads those v-heads read), so the rank
    writes its part of ``output`` and ``new_state`` in place and nothing is copied
    except each run's small ``cu_seqlens``.  ``seqlens`` are the host-side lengths the
    plan was made from; ``state`` may be None (zeros)."""
    import torch

    lens = [int(x) for x in seqlens]
    HQ, HV = q.shape[1], v.shape[1]
    if HV % HQ:
        raise ValueError(f"{HV} v-heads do not map onto {HQ} q/k heads")
    ratio = HV // HQ
    lo, hi = shard.head_lo, shard.head_hi
    if lo % ratio or hi % ratio:
        raise ValueError(f"v-head range [{lo}, {hi}) splits a q/k head (GVA ratio {ratio})")
    starts = [0]
    for n in lens:
        starts.append(starts[-1] + n)
    runs = []
    for i in sorted(shard.seqs):
        if runs and runs[-1][1] == i:
            runs[-1][1] = i + 1
        else:
            runs.append([i, i + 1])
    cu_dtype = cu_dtype or torch.int32
    calls = []
    for s0, s1 in runs:
        t0, t1 = starts[s0], starts[s1]
        cu = torch.tensor([x - t0 for x in starts[s0:s1 + 1]], dtype=cu_dtype, device=q.device)
        calls.append(dict(
            q=q[t0:t1, lo // ratio:hi // ratio], k=k[t0:t1, lo // ratio:hi // ratio], v=v[t0:t1, lo:hi],
            state=None if state is None else state[s0:s1, lo:hi], A_log=A_log[lo:hi], a=a[t0:t1, lo:hi],
            dt_bias=dt_bias[lo:hi], b=b[t0:t1, lo:hi], cu_seqlens=cu, output=output[t0:t1, lo:hi],
            new_state=new_state[s0:s1, lo:hi]))
    return calls


def gather_to_rank0(tensor, group=None):
    """Optional NCCL gather of equally-shaped per-rank outputs onto rank 0
    (``all_gather`` over NVLink; never on the timed hot path).  Returns the list
    of tensors on rank 0 and None elsewhere."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    parts = [torch.empty_like(tensor) for _ in range(world)]
    dist.all_gather(parts, tensor.contiguous(), group=group)
    return parts if dist.get_rank(group) == 0 else None
