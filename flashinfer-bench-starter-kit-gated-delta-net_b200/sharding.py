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
