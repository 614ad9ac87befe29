"""Multi-GPU work split (host logic) and its world_size-2 gloo exercise. CPU only."""
from __future__ import annotations

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def test_batch_slices_cover_batch(gdn):
    for B in (1, 7, 64, 1024):
        for world in (1, 2, 4, 8):
            spans = [gdn.sharding.batch_slice(B, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == B
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1


def test_prefill_plan_whole_sequences_balanced(gdn):
    lens = gdn.workloads.varlen_seqlens()
    for world in (1, 2, 4, 8):
        plan = gdn.sharding.plan_prefill(lens, 32, world)
        seqs = sorted(i for s in plan for i in s.seqs)
        assert seqs == list(range(len(lens)))
        loads = [s.tokens for s in plan]
        assert max(loads) <= sum(lens) / world + max(lens)


def test_prefill_plan_head_split_for_few_sequences(gdn):
    plan = gdn.sharding.plan_prefill([32768] * 8, 32, 16)  # fewer sequences than ranks
    assert [(s.head_lo, s.head_hi) for s in plan][:2] == [(0, 2), (2, 4)]
    assert all(s.seqs == list(range(8)) for s in plan)
    with pytest.raises(ValueError):
        gdn.sharding.plan_prefill([10] * 2, 32, 3)


def _gather_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    from __graft_entry__ import load_package

    gdn = load_package()
    s, e = gdn.sharding.batch_slice(10, world, rank)
    local = torch.arange(s, e, dtype=torch.float32)
    local = torch.nn.functional.pad(local, (0, 5 - local.numel()), value=-1)
    parts = gdn.sharding.gather_to_rank0(local)
    if rank == 0:
        q.put(torch.cat(parts).tolist())
    dist.barrier()
    dist.destroy_process_group()


def test_gather_to_rank0_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [x for x in got if x >= 0] == list(range(10))


def test_prefill_shard_calls_cover_every_token_and_head_once(gdn):
    """The views a rank's share becomes (no copies but each run's cu_seqlens) tile the
    call's (token, v-head) and (sequence, v-head) grids exactly once over the ranks,
    for whole-sequence shards and for v-head-pair shards.  CPU tensors: views only."""
    for lens, world in (([70, 5, 300, 64, 1], 2), ([70, 5, 300, 64, 1], 4), ([900, 257], 4), ([33], 8)):
        T, N = sum(lens), len(lens)
        q = torch.zeros(T, 16, 128, dtype=torch.bfloat16)
        v = torch.zeros(T, 32, 128, dtype=torch.bfloat16)
        ab = torch.zeros(T, 32, dtype=torch.bfloat16)
        par = torch.zeros(32)
        out = torch.zeros(T, 32, 128, dtype=torch.bfloat16)
        ns = torch.zeros(N, 32, 4, 4)
        seen_tok = torch.zeros(T, 32, dtype=torch.int32)
        seen_seq = torch.zeros(N, 32, dtype=torch.int32)
        for shard in gdn.sharding.plan_prefill(lens, 32, world):
            for c in gdn.sharding.prefill_shard_calls(shard, lens, q, q, v, None, par, ab, par, ab, out, ns):
                t0 = (c["output"].data_ptr() - out.data_ptr()) // (out.stride(0) * 2)
                h0 = (c["v"].data_ptr() - v.data_ptr()) // 2 % (32 * 128) // 128
                nt, nh = c["output"].shape[0], c["output"].shape[1]
                assert c["q"].shape[1] * 2 == nh and c["a"].shape == (nt, nh) and c["A_log"].shape == (nh,)
                assert int(c["cu_seqlens"][-1]) == nt and c["cu_seqlens"].dtype == torch.int32
                seen_tok[t0:t0 + nt, h0:h0 + nh] += 1
                s0 = (c["new_state"].data_ptr() - ns.data_ptr()) // (ns.stride(0) * 4)
                seen_seq[s0:s0 + c["new_state"].shape[0], h0:h0 + nh] += 1
        assert bool((seen_tok == 1).all()) and bool((seen_seq == 1).all()), (lens, world)
