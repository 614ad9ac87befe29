"""The decode and pooled-decode launches inside a CUDA graph (the serving form of a
decode loop, and how bench.py times them): a captured sequence of steps replays to
exactly the results of the same steps launched directly."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def to_dev(inp):
    return {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}


def test_decode_steps_replay_bit_exact(gdn):
    """Three chained decode steps (each step's new state is the next step's state,
    ping-pong buffers) captured once and replayed equal the eager steps bit for bit."""
    inp = to_dev(gdn.workloads.decode_inputs(5, seed=31))
    B = inp["q"].shape[0]
    out = torch.empty(B, 1, 32, 128, dtype=torch.bfloat16, device="cuda")
    st = [inp["state"].clone(), torch.empty_like(inp["state"])]

    def steps(o, s):
        for i in range(3):
            gdn.kernel_decode.run_dps(inp["q"], inp["k"], inp["v"], s[i % 2], inp["A_log"], inp["a"], inp["dt_bias"],
                                      inp["b"], inp["scale"], o, s[(i + 1) % 2])

    steps(out, st)  # eager (also the warm-up before capture)
    torch.cuda.synchronize()
    eager_out, eager_state = out.clone(), st[1].clone()

    st[0].copy_(inp["state"])
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        steps(out, st)
    out.zero_()
    st[1].zero_()
    st[0].copy_(inp["state"])
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager_out)
    assert torch.equal(st[1], eager_state)


def test_pooled_decode_replay_bit_exact(gdn):
    """A pooled multi-token decode (in place on the pool) captured and replayed from the
    same pool contents equals the eager call bit for bit."""
    B, T, P = 4, 3, 9
    inp = to_dev(gdn.workloads.prefill_inputs([T] * B, seed=5))
    q = inp["q"].view(B, T, 16, 128)
    k = inp["k"].view(B, T, 16, 128)
    v = inp["v"].view(B, T, 32, 128)
    a = inp["a"].view(B, T, 32)
    b = inp["b"].view(B, T, 32)
    gen = torch.Generator().manual_seed(3)
    pool0 = (torch.randn(P, 32, 128, 128, generator=gen) * 0.05).cuda()
    idx = torch.tensor([7, 2, -1, 4], dtype=torch.int32, device="cuda")
    out = torch.empty(B, T, 32, 128, dtype=torch.bfloat16, device="cuda")
    pool = pool0.clone()

    def call():
        gdn.kernel_mtp.run_dps(q, k, v, pool, idx, inp["A_log"], a, inp["dt_bias"], b, None, out, pool)

    call()
    torch.cuda.synchronize()
    eager_out, eager_pool = out.clone(), pool.clone()
    pool.copy_(pool0)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        call()
    out.zero_()
    pool.copy_(pool0)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager_out)
    assert torch.equal(pool, eager_pool)
