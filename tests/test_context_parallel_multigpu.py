"""Context-parallel prefill over NCCL ranks, one per GPU (2 or more B200s): each rank
holds its token ranges of the sequences, exchanges affine state maps once and returns
its outputs and the final states; compared on every rank with the single-GPU prefill
of the whole batch (bf16 outputs atol = rtol = 1e-2, states 1e-3 relative).  Skipped
with fewer than 2 GPUs.  NVLS is off (plain NCCL)."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import state_close

pytestmark = pytest.mark.gpu
LENS = [4096 + 100, 1000]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from __graft_entry__ import load_package

    gdn = load_package()
    cp = gdn.context_parallel
    inp = gdn.workloads.prefill_inputs(LENS, seed=350, device=f"cuda:{rank}")
    loc = cp.local_inputs(inp, world, rank)
    out, final = cp.prefill_context_parallel(loc["q"], loc["k"], loc["v"], loc["state"], loc["A_log"], loc["a"],
                                             loc["dt_bias"], loc["b"], loc["cu_seqlens"], loc["scale"])
    o_all, s_all = gdn.kernel_prefill.run(**inp)  # the whole batch on this GPU
    torch.cuda.synchronize()
    ranges = cp.split_ranges(LENS, world)[rank]
    cu = np.concatenate([[0], np.cumsum(LENS)])
    idx = np.concatenate([np.arange(cu[i] + lo, cu[i] + hi) for i, (lo, hi) in enumerate(ranges)])
    want = o_all[torch.from_numpy(idx).cuda()].float()
    o_err = float(((out.float() - want).abs() - 1e-2 * want.abs()).max())  # atol = rtol = 1e-2
    ok, s_err = state_close(final.cpu().numpy(), s_all.cpu().numpy(), 1e-3)
    q.put((rank, o_err, ok, s_err))
    dist.barrier()
    dist.destroy_process_group()


def test_context_parallel_nccl_ranks():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    world = min(world, 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, o_err, ok, s_err in res:
        assert o_err <= 1e-2, (rank, o_err)
        assert ok, (rank, s_err)
