"""Context parallelism across ranks (``context_parallel``): the range split, and the
exchange protocol (affine state maps, one all_gather, fold, rerun, broadcast) on
world_size 2 and 3 gloo ranks on CPU.  The per-rank computations are the CPU oracle
here (the CUDA kernels' maps are checked against it in the GPU tests), so these
tests pin the algebra and the collective steps; the oracle's full-sequence prefill
is the reference.  Tolerances: bf16 outputs atol = rtol = 1e-2, states 1e-3 relative."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import state_close
from oracle import gdn_oracle as ref

LENS = [300, 70, 0, 513]  # 2 chunks and a tail, sub-chunk, empty, 8 chunks and a tail
HQ, HV = 2, 4


def test_split_ranges_cover_each_sequence(gdn):
    cp = gdn.context_parallel
    lens = [0, 1, 37, 64, 65, 700, 4096, 130]
    for weight in (1.0, cp.FIRST_RANK_WEIGHT, 3.0):
        for world in (1, 2, 3, 4, 8):
            ranges = cp.split_ranges(lens, world, weight)
            for i, L in enumerate(lens):
                spans = [ranges[r][i] for r in range(world)]
                assert spans[0][0] == 0 and spans[-1][1] == L
                assert all(x[1] == y[0] for x, y in zip(spans, spans[1:]))
                assert all(s[0] % 64 == 0 for s in spans)  # every range starts on a chunk boundary
                sizes = [(e - s + 63) // 64 for s, e in spans]
                if weight == 1.0:
                    assert max(sizes) - min(sizes) <= 1
    # weighted: rank 0 holds first_weight times the chunks of each other rank (to a chunk)
    r = cp.split_ranges([64 * 380], 4, 0.8)
    assert [(hi - lo) // 64 for lo, hi in (x[0] for x in r)] == [80, 100, 100, 100]


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _oracle_ops(cp):
    def prefill(q, k, v, state, A_log, a, dt_bias, b, cu, scale):
        o, s = ref.prefill(_bits(q), _bits(k), _bits(v), None if state is None else state.numpy(), A_log.numpy(),
                           _bits(a), dt_bias.numpy(), _bits(b), cu.numpy(), scale)
        return torch.from_numpy(ref.bf16_bits_to_f32(o)), torch.from_numpy(np.ascontiguousarray(s))

    def state_map(q, k, v, A_log, a, dt_bias, b, cu):
        N, H = cu.shape[0] - 1, v.shape[1]
        eye = np.broadcast_to(np.eye(128, dtype=np.float32), (N, H, 128, 128)).copy()
        _, m = ref.prefill(_bits(q), _bits(k), np.zeros_like(_bits(v)), eye, A_log.numpy(), _bits(a),
                           dt_bias.numpy(), _bits(b), cu.numpy(), None)
        _, c = ref.prefill(_bits(q), _bits(k), _bits(v), None, A_log.numpy(), _bits(a), dt_bias.numpy(), _bits(b),
                           cu.numpy(), None)
        return torch.from_numpy(np.ascontiguousarray(m)), torch.from_numpy(np.ascontiguousarray(c))

    def affine(q, k, v, A_log, a, dt_bias, b, cu, scale):
        # the range's map now; its outputs once the incoming state is known (a rerun here)
        m, c = state_map(q, k, v, A_log, a, dt_bias, b, cu)
        return (q, k, v, A_log, a, dt_bias, b, cu, scale), m, c

    def finish(handle, prev):
        q, k, v, A_log, a, dt_bias, b, cu, scale = handle
        s_in = torch.zeros_like(prev[0, 0])
        for j in range(prev.shape[0]):  # the fold of the preceding ranges' maps
            s_in = torch.matmul(s_in, prev[j, 0]) + prev[j, 1]
        return prefill(q, k, v, s_in, A_log, a, dt_bias, b, cu, scale)

    return cp.Ops(prefill=prefill, affine=affine, finish=finish)


def _cp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from __graft_entry__ import load_package

    gdn = load_package()
    cp = gdn.context_parallel
    inp = gdn.workloads.prefill_inputs(LENS, num_qk_heads=HQ, num_v_heads=HV, seed=77)
    loc = cp.local_inputs(inp, world, rank)
    out, final = cp.prefill_context_parallel(loc["q"], loc["k"], loc["v"], loc["state"], loc["A_log"], loc["a"],
                                             loc["dt_bias"], loc["b"], loc["cu_seqlens"], loc["scale"],
                                             ops=_oracle_ops(cp))
    q.put((rank, out.numpy(), final.numpy()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_context_parallel_gloo_matches_whole_sequences(gdn, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + (os.getpid() + 7 * world) % 1000
    procs = [ctx.Process(target=_cp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {r: (o, f) for r, o, f in (q.get(timeout=600) for _ in range(world))}
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    inp = gdn.workloads.prefill_inputs(LENS, num_qk_heads=HQ, num_v_heads=HV, seed=77)
    o_ref, s_ref = ref.prefill(_bits(inp["q"]), _bits(inp["k"]), _bits(inp["v"]), inp["state"].numpy(),
                               inp["A_log"].numpy(), _bits(inp["a"]), inp["dt_bias"].numpy(), _bits(inp["b"]),
                               inp["cu_seqlens"].numpy(), inp["scale"])
    o_ref = ref.bf16_bits_to_f32(o_ref)
    # reassemble the outputs in global token order
    ranges = gdn.context_parallel.split_ranges(LENS, world)
    cu = np.concatenate([[0], np.cumsum(LENS)])
    out = np.zeros_like(o_ref)
    for r in range(world):
        pos = 0
        for i, (lo, hi) in enumerate(ranges[r]):
            out[cu[i] + lo:cu[i] + hi] = got[r][0][pos:pos + hi - lo]
            pos += hi - lo
    np.testing.assert_allclose(out, o_ref, atol=1e-2, rtol=1e-2)
    for r in range(world):  # every rank returns the sequences' final state
        ok, err = state_close(got[r][1], s_ref, 1e-3)
        assert ok, (r, err)
