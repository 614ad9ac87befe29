"""Context-parallel chunked prefill (each sequence's chunks split into segments that
run on separate SMs: per-segment affine state maps, their composition, then the
segments rerun from their initial states) against the CPU oracle, through the C ABI.
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
    records = (T // 64 + 1 + 1) * 32 * 17664
    assert gdn.kernel_prefill.workspace_size(1, T, 16, 32) > records
    assert gdn.kernel_prefill.workspace_size(1, T, 16, 32, segments=1) == records
    out, ns = gdn.kernel_prefill.run(**to_dev(inp))
    torch.cuda.synchronize()
    o_ref, s_ref = oracle_prefill(inp)
    assert_match(out, ns, o_ref, s_ref)
    assert gdn._lib.device_error() == 0


def test_segments_in_place_without_allocation(gdn):
    """In-place state update through the static-scratch entry point, 4 segments."""
    lens = [1500, 900]
    inp = gdn.workloads.prefill_inputs(lens, seed=320)
    o_ref, s_ref = oracle_prefill(inp)
    dev = to_dev(inp)
    state = dev["state"].clone()
    out = torch.empty(sum(lens), 32, 128, dtype=torch.bfloat16, device="cuda")
    gdn.kernel_prefill.run_dps(dev["q"], dev["k"], dev["v"], state, dev["A_log"], dev["a"], dev["dt_bias"],
                               dev["b"], dev["cu_seqlens"], dev["scale"], out, state, no_alloc=True, segments=4)
    torch.cuda.synchronize()
    assert_match(out, state, o_ref, s_ref)
