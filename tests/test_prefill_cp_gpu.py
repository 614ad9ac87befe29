"""Context-parallel chunked prefill (each sequence's chunks split into segments that
run on separate SMs: segment 0 from the initial state, the later segments' affine state
maps and homogeneous outputs, the maps' composition, then the later segments' outputs
corrected by their initial states) against the CPU oracle, through the C ABI.
Tolerances as for every prefill: bf16 outputs atol = rtol = 1e-2, final states
within 1e-3 relative."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import state_close
from oracle import c_oracle
from oracle import gdn_oracle as ref

pytestmark = pytest.mark.gpu
OUT_TOL = dict(atol=1e-2, rtol=1e-2)


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def to_dev(inp):
    return {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}


def oracle_prefill(inp):
    st = inp["state"]
    return c_oracle.prefill(bits(inp["q"]), bits(inp["k"]), bits(inp["v"]),
                            None if st is None else st.cpu().numpy(), inp["A_log"].cpu().numpy(),
                            bits(inp["a"]), inp["dt_bias"].cpu().numpy(), bits(inp["b"]),
                            inp["cu_seqlens"].cpu().numpy(), inp["scale"])


def assert_match(out, new_state, o_ref_bits, s_ref):
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.bf16_bits_to_f32(o_ref_bits), **OUT_TOL)
    ok, err = state_close(new_state.cpu().numpy(), s_ref, 1e-3)
    assert ok, f"state rel err {err}"


@pytest.mark.parametrize("segments", [2, 3, 5])
def test_forced_segments_match_oracle(gdn, segments):
    """Empty, sub-chunk, partial-last-chunk and sequences shorter than the segment
    count (empty segments) in one call."""
    lens = [0, 37, 700, 2061, 192]
    inp = gdn.workloads.prefill_inputs(lens, seed=300 + segments)
    dev = to_dev(inp)
    out, ns = gdn.kernel_prefill.run(**dev, segments=segments)
    torch.cuda.synchronize()
    o_ref, s_ref = oracle_prefill(inp)
    assert_match(out, ns, o_ref, s_ref)
    assert torch.equal(ns[0], dev["state"][0])  # empty sequence: state passes through
    assert gdn._lib.device_error() == 0
    # the single-chain kernel on the same inputs agrees to fp32 rounding of the map products
    out1, ns1 = gdn.kernel_prefill.run(**dev, segments=1)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.float().cpu().numpy(), out1.float().cpu().numpy(), atol=1e-2, rtol=1e-2)
    ok, err = state_close(ns.cpu().numpy(), ns1.cpu().numpy(), 1e-4)
    assert ok, err


def test_automatic_segments_one_long_sequence(gdn):
    """One sequence, 32 v-heads: 32 chains would leave most of the 148 SMs idle, so
    the library splits the sequence (its workspace grows by the segment scratch)."""
    T = 64 * 70 + 9
    inp = gdn.workloads.prefill_inputs([T], seed=310)
    records = (T // 64 + 1 + 1) * 32 * 11008
    assert gdn.kernel_prefill.workspace_size(1, T, 16, 32) > records
    assert gdn.kernel_prefill.workspace_size(1, T, 16, 32, segments=1) == records
    out, ns = gdn.kernel_prefill.run(**to_dev(inp))
    torch.cuda.synchronize()
    o_ref, s_ref = oracle_prefill(inp)
    assert_match(out, ns, o_ref, s_ref)
    assert gdn._lib.device_error() == 0


def test_segments_in_place_without_allocation(gdn):
    """In-place state update through the static-scratch entry point, 3 segments."""
    lens = [1500, 900]
    inp = gdn.workloads.prefill_inputs(lens, seed=320)
    o_ref, s_ref = oracle_prefill(inp)
    dev = to_dev(inp)
    state = dev["state"].clone()
    out = torch.empty(sum(lens), 32, 128, dtype=torch.bfloat16, device="cuda")
    gdn.kernel_prefill.run_dps(dev["q"], dev["k"], dev["v"], state, dev["A_log"], dev["a"], dev["dt_bias"],
                               dev["b"], dev["cu_seqlens"], dev["scale"], out, state, no_alloc=True, segments=3)
    torch.cuda.synchronize()
    assert_match(out, state, o_ref, s_ref)


def _oracle_map(inp):
    N, H = inp["cu_seqlens"].shape[0] - 1, inp["v"].shape[1]
    eye = np.broadcast_to(np.eye(128, dtype=np.float32), (N, H, 128, 128)).copy()
    args = (inp["A_log"].cpu().numpy(), bits(inp["a"]), inp["dt_bias"].cpu().numpy(), bits(inp["b"]),
            inp["cu_seqlens"].cpu().numpy(), None)
    _, m = c_oracle.prefill(bits(inp["q"]), bits(inp["k"]), np.zeros_like(bits(inp["v"])), eye, *args)
    _, c = c_oracle.prefill(bits(inp["q"]), bits(inp["k"]), bits(inp["v"]), None, *args)
    return m, c


@pytest.mark.parametrize("slow_decay,segments", [(False, 0), (True, 0), (True, 3)])
def test_state_map_matches_oracle_and_is_affine(gdn, slow_decay, segments):
    """M = the range from the identity with v = 0, C = the range from zero; and the
    prefill from any state S ends in S M + C.  With the benchmark gates the state
    forgets its start within tens of tokens (M falls to 1e-18 .. 1e-38 on the short
    ranges), so M is checked to 1e-3 of its size plus 1e-6 absolute (S M then errs
    by far less than the 1e-3 state tolerance); with slow decay (A_log = -6) M stays
    O(1) and the check is relative."""
    lens = [0, 37, 700, 130]
    inp = gdn.workloads.prefill_inputs(lens, seed=330)
    if slow_decay:
        inp["A_log"] = torch.full_like(inp["A_log"], -6.0)
    dev = to_dev(inp)
    M, C = gdn.kernel_prefill.state_map(dev["q"], dev["k"], dev["v"], dev["A_log"], dev["a"], dev["dt_bias"],
                                        dev["b"], dev["cu_seqlens"], segments=segments)
    torch.cuda.synchronize()
    m_ref, c_ref = _oracle_map(inp)
    ok, err = state_close(C[1:].cpu().numpy(), c_ref[1:], 1e-3)
    assert ok, err
    dm = np.abs(M.cpu().numpy() - m_ref).reshape(len(lens), 32, -1).max(-1)
    scale = np.abs(m_ref).reshape(len(lens), 32, -1).max(-1)
    assert (dm <= 1e-3 * scale + 1e-6).all(), float((dm / np.maximum(scale, 1e-30)).max())
    if slow_decay:
        assert scale[1:].min() > 1e-3  # the maps are far from zero here (1e-2 .. 1 by head)
    assert torch.equal(M[0], torch.eye(128, device="cuda").expand_as(M[0])) and not C[0].any()  # empty range
    _, fin = gdn.kernel_prefill.run(**dev, segments=1)
    comp = torch.matmul(dev["state"], M) + C
    torch.cuda.synchronize()
    ok, err = state_close(comp.cpu().numpy(), fin.cpu().numpy(), 1e-4)
    assert ok, err


def test_state_map_automatic_segments_one_long_sequence(gdn):
    """One sequence, 32 v-heads: the map is computed in segments (the workspace grows
    by their maps), multiplied on the GPU; slow decay keeps M far from zero."""
    T = 64 * 40 + 5
    inp = gdn.workloads.prefill_inputs([T], seed=335)
    inp["A_log"] = torch.full_like(inp["A_log"], -6.0)
    lib = gdn._lib.library()
    records = (T // 64 + 2) * 32 * 11008
    assert lib.gdn_prefill_workspace_size(1, T, 16, 32, 128, gdn._lib.GDN_FLAG_STATE_MAP) > records
    dev = to_dev(inp)
    M, C = gdn.kernel_prefill.state_map(dev["q"], dev["k"], dev["v"], dev["A_log"], dev["a"], dev["dt_bias"],
                                        dev["b"], dev["cu_seqlens"])
    M1, C1 = gdn.kernel_prefill.state_map(dev["q"], dev["k"], dev["v"], dev["A_log"], dev["a"], dev["dt_bias"],
                                          dev["b"], dev["cu_seqlens"], segments=1)
    torch.cuda.synchronize()
    m_ref, c_ref = _oracle_map(inp)
    for got in ((M, C), (M1, C1)):
        for g_, w_ in zip(got, (m_ref, c_ref)):
            ok, err = state_close(g_.cpu().numpy(), w_, 1e-3)
            assert ok, err


def test_context_parallel_steps_on_one_gpu(gdn):
    """The three ranks of a context-parallel prefill emulated on one device with the
    CUDA operators (rank 0's prefill, the other ranks' affine passes, their finishes from
    the gathered maps) against the oracle's whole sequences."""
    cp = gdn.context_parallel
    ops = cp.cuda_ops()
    lens, world = [2000, 513, 64], 3
    inp = gdn.workloads.prefill_inputs(lens, seed=340)
    dev = to_dev(inp)
    locs = [cp.local_inputs(dev, world, r) for r in range(world)]
    keys = ("q", "k", "v")
    gate = lambda L: (L["A_log"], L["a"], L["dt_bias"], L["b"], L["cu_seqlens"])  # noqa: E731
    outs = [None] * world
    outs[0], s = ops.prefill(*(locs[0][x] for x in keys), dev["state"], *gate(locs[0]), dev["scale"])
    affine = [None] + [ops.affine(*(locs[r][x] for x in keys), *gate(locs[r]), dev["scale"])
                       for r in range(1, world)]
    pairs = torch.stack([torch.stack([torch.zeros_like(s), s])] +
                        [torch.stack([affine[r][1], affine[r][2]]) for r in range(1, world)])
    for r in range(1, world):
        outs[r], s_r = ops.finish(affine[r][0], pairs[:r])  # folds the preceding ranges' maps on the GPU
    torch.cuda.synchronize()
    o_ref, s_ref = oracle_prefill(inp)
    o_ref = ref.bf16_bits_to_f32(o_ref)
    ranges = cp.split_ranges(lens, world)
    cu = np.concatenate([[0], np.cumsum(lens)])
    out = np.zeros_like(o_ref)
    for r in range(world):
        pos, o = 0, outs[r].float().cpu().numpy()
        for i, (lo, hi) in enumerate(ranges[r]):
            out[cu[i] + lo:cu[i] + hi] = o[pos:pos + hi - lo]
            pos += hi - lo
    np.testing.assert_allclose(out, o_ref, **OUT_TOL)
    ok, err = state_close(s_r.cpu().numpy(), s_ref, 1e-3)
    assert ok, err


def _cut(inp, cuts):
    """Head [0, x) and tail [x, L) of every sequence as two prefill input dicts."""
    cu = inp["cu_seqlens"].cpu().tolist()
    head_idx, tail_idx, head_cu, tail_cu = [], [], [0], [0]
    for i, x in enumerate(cuts):
        lo, hi = cu[i], cu[i + 1]
        head_idx.append(torch.arange(lo, lo + x))
        tail_idx.append(torch.arange(lo + x, hi))
        head_cu.append(head_cu[-1] + x)
        tail_cu.append(tail_cu[-1] + hi - lo - x)
    parts = []
    for idx, c in ((torch.cat(head_idx), head_cu), (torch.cat(tail_idx), tail_cu)):
        d = dict(inp)
        idx = idx.to(inp["q"].device)
        for key in ("q", "k", "v", "a", "b"):
            d[key] = inp[key].index_select(0, idx).contiguous()
        d["cu_seqlens"] = torch.tensor(c, dtype=inp["cu_seqlens"].dtype, device=inp["cu_seqlens"].device)
        parts.append((d, idx))
    return parts


@pytest.mark.parametrize("segments", [0, 1, 3])
def test_range_affine_finish_matches_whole_sequences(gdn, segments):
    """A later token range of every sequence run as ``range_affine`` (its outputs from a
    zero state and its map, before the state entering it is known) and ``range_finish``
    (given that state): the outputs and final states of the whole-sequence prefill, and
    the map of ``state_map``.  Empty, sub-chunk and partial-chunk ranges; automatic and
    forced segment counts; the finish in place."""
    lens = [0, 37, 700, 2061, 192, 1500]
    inp = to_dev(gdn.workloads.prefill_inputs(lens, seed=360 + segments))
    o_all, s_all = gdn.kernel_prefill.run(**inp, segments=1)
    (head, _), (tail, tail_idx) = _cut(inp, [64 * ((L // 64) // 2) for L in lens])
    _, s_mid = gdn.kernel_prefill.run(**head, segments=1)
    args = [tail[k] for k in ("q", "k", "v", "A_log", "a", "dt_bias", "b", "cu_seqlens", "scale")]
    h = gdn.kernel_prefill.range_affine(*args, segments=segments)
    m_ref, c_ref = gdn.kernel_prefill.state_map(*args[:8], segments=1)
    torch.cuda.synchronize()
    # M is dimensionless (identity scale); where the decay has all but emptied it, the segmented
    # and single-chain products differ relative to its size but not to the identity's
    assert float((h.map_m - m_ref).abs().max()) <= 1e-4
    ok, err = state_close(h.map_c.cpu().numpy(), c_ref.cpu().numpy(), 1e-3)
    assert ok, err
    composed = torch.matmul(s_mid, h.map_m) + h.map_c  # what the other ranks' exchange uses
    ok, err = state_close(composed.cpu().numpy(), s_all.cpu().numpy(), 1e-3)
    assert ok, err
    s_in = s_mid.clone()
    out, s_end = gdn.kernel_prefill.range_finish(h, s_in, new_state=s_in)  # in place
    torch.cuda.synchronize()
    assert s_end is s_in
    np.testing.assert_allclose(out.float().cpu().numpy(), o_all[tail_idx].float().cpu().numpy(), **OUT_TOL)
    ok, err = state_close(s_end.cpu().numpy(), s_all.cpu().numpy(), 1e-3)
    assert ok, err
    assert torch.equal(s_end[0], s_mid[0])  # empty sequence: the state passes through
    assert gdn._lib.device_error() == 0
