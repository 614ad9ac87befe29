"""Varlen prefill parity on the GPU (through the C ABI) against the reference
kernel's golden vectors and the CPU oracle.  Tolerances as in the decode tests:
bf16 output atol = rtol = 1e-2; final fp32 state within 1e-3 relative."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden, state_close
from oracle import c_oracle
from oracle import gdn_oracle as ref

pytestmark = pytest.mark.gpu
OUT_TOL = dict(atol=1e-2, rtol=1e-2)
STATE_RTOL = 1e-3


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def to_dev(inp):
    return {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}


def oracle_prefill(inp, impl=ref, **kw):
    st = inp["state"]
    return impl.prefill(bits(inp["q"]), bits(inp["k"]), bits(inp["v"]),
                        None if st is None else st.cpu().numpy(), inp["A_log"].cpu().numpy(),
                        bits(inp["a"]), inp["dt_bias"].cpu().numpy(), bits(inp["b"]),
                        inp["cu_seqlens"].cpu().numpy(), inp["scale"], **kw)


def assert_match(out, new_state, o_ref_bits, s_ref):
    o = out.float().cpu().numpy()
    np.testing.assert_allclose(o, ref.bf16_bits_to_f32(o_ref_bits), **OUT_TOL)
    ok, err = state_close(new_state.cpu().numpy(), s_ref, STATE_RTOL)
    assert ok, f"state rel err {err}"


def test_golden_reference_kernel(gdn):
    g = load_golden("prefill_qk4v8_lens1-0-70")
    tb = lambda x: torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()  # noqa: E731
    state = torch.from_numpy(ref.bf16_bits_to_f32(g["state"])).cuda()
    out, ns = gdn.kernel_prefill.run(tb(g["q"]), tb(g["k"]), tb(g["v"]), state,
                                     torch.from_numpy(g["A_log"]).cuda(), tb(g["a"]),
                                     torch.from_numpy(g["dt_bias"]).cuda(), tb(g["b"]),
                                     torch.from_numpy(g["cu_seqlens"]).cuda(), None)
    torch.cuda.synchronize()
    assert_match(out, ns, g["out_triton"], g["new_state_triton"])
    # empty sequence: initial state passes through unchanged
    assert torch.equal(ns[1], state[1])


@pytest.mark.parametrize("lens", [[1], [64], [65], [1, 0, 63, 64, 65, 130], [0, 0], [200, 3, 129]])
def test_random_varlen(gdn, lens):
    inp = gdn.workloads.prefill_inputs(lens, seed=sum(lens) + len(lens))
    out, ns = gdn.kernel_prefill.run(**to_dev(inp))
    o_ref, s_ref = oracle_prefill(inp)
    assert_match(out, ns, o_ref, s_ref)
    assert gdn._lib.device_error() == 0


def test_int64_cu_seqlens_zero_state(gdn):
    inp = gdn.workloads.prefill_inputs([70, 5], seed=31, cu_dtype=torch.int64)
    inp["state"] = None
    out, ns = gdn.kernel_prefill.run(**to_dev(inp))
    o_ref, s_ref = oracle_prefill(inp)
    assert_match(out, ns, o_ref, s_ref)


def test_qk_l2norm_and_gva_ratio_4(gdn):
    inp = gdn.workloads.prefill_inputs([40, 77], num_qk_heads=8, seed=32)
    inp["q"] = (inp["q"].float() * 2.0).bfloat16()
    out, ns = gdn.kernel_prefill.run(**to_dev(inp), use_qk_l2norm=True)
    o_ref, s_ref = oracle_prefill(inp, use_qk_l2norm=True)
    assert_match(out, ns, o_ref, s_ref)


def test_in_place_state(gdn):
    inp = gdn.workloads.prefill_inputs([33, 96], seed=33)
    d = to_dev(inp)
    st = d["state"].clone()
    out = torch.empty(129, 32, 128, dtype=torch.bfloat16, device="cuda")
    gdn.kernel_prefill.run_dps(d["q"], d["k"], d["v"], st, d["A_log"], d["a"], d["dt_bias"], d["b"],
                               d["cu_seqlens"], None, out, st)
    o_ref, s_ref = oracle_prefill(inp)
    assert_match(out, st, o_ref, s_ref)


def test_bad_cu_seqlens_sets_device_error(gdn):
    inp = to_dev(gdn.workloads.prefill_inputs([8, 8], seed=34))
    inp["cu_seqlens"] = torch.tensor([0, 12, 9], dtype=torch.int32, device="cuda")  # not monotone
    gdn._lib.device_error(clear=True)
    gdn.kernel_prefill.run(**inp)
    assert gdn._lib.device_error(clear=True) & gdn._lib.GDN_DEVERR_BAD_SEQLENS


# ----------------------------------------------------------------------------- chunked tensor-core path
@pytest.mark.parametrize("lens", [[63], [127, 128, 129], [256, 0, 1, 191], [1000]])
def test_chunked_matches_oracle_at_chunk_boundaries(gdn, lens):
    inp = gdn.workloads.prefill_inputs(lens, seed=40 + len(lens))
    out, ns = gdn.kernel_prefill.run(**to_dev(inp))
    o_ref, s_ref = oracle_prefill(inp, impl=c_oracle)
    assert_match(out, ns, o_ref, s_ref)
    assert gdn._lib.device_error() == 0


def test_chunked_long_memory_gates(gdn):
    """Decays close to 1 (long memory): the chunked path's bf16 operand splits must
    keep the final state within tolerance over many chunks."""
    inp = gdn.workloads.prefill_inputs([700, 1500], seed=41)
    inp["dt_bias"] = inp["dt_bias"] - 6.0   # softplus(a + dt) ~ 1e-3  ->  g ~ 0.99
    inp["A_log"] = inp["A_log"] * 0.2
    out, ns = gdn.kernel_prefill.run(**to_dev(inp))
    o_ref, s_ref = oracle_prefill(inp, impl=c_oracle)
    assert_match(out, ns, o_ref, s_ref)


def test_chunked_equals_serial_kernel(gdn):
    inp = to_dev(gdn.workloads.prefill_inputs([300, 64, 5, 0, 77], seed=42))
    o1, s1 = gdn.kernel_prefill.run(**inp)
    o2, s2 = gdn.kernel_prefill.run(**inp, serial=True)
    torch.cuda.synchronize()
    np.testing.assert_allclose(o1.float().cpu().numpy(), o2.float().cpu().numpy(), **OUT_TOL)
    ok, err = state_close(s1.cpu().numpy(), s2.cpu().numpy(), STATE_RTOL)
    assert ok, err


def test_golden_reference_kernel_16_32_heads(gdn):
    """BASELINE.json's head counts (16 q/k, 32 v heads) over several chunks (200 tokens:
    3 full chunks and 8 tokens; an empty sequence; 65 tokens) against the reference kernel."""
    from test_oracle import qk16v32_prefill_case

    g, (q, k, v, a, b, A_log, dt_bias, state, cu) = qk16v32_prefill_case()
    dev = lambda t: t.cuda()  # noqa: E731
    out, ns = gdn.kernel_prefill.run(dev(q), dev(k), dev(v), dev(state), dev(A_log), dev(a), dev(dt_bias), dev(b),
                                     dev(cu), None)
    torch.cuda.synchronize()
    assert_match(out, ns[:, torch.from_numpy(g["stored_heads"]).cuda()], g["out_triton"], g["new_state_triton"])
    assert torch.equal(ns[1], state[1].cuda())


# ----------------------------------------------------------------------------- in-kernel q/k L2 norm
def _unnormalised(inp, seed):
    """q and k rows with random norms in [0.3, 3] (bf16), so the normalisation matters."""
    g = torch.Generator().manual_seed(seed)
    for key in ("q", "k"):
        x = inp[key].float()
        scale = 0.3 + 2.7 * torch.rand(x.shape[0], x.shape[1], 1, generator=g)
        inp[key] = (x * scale).bfloat16()
    return inp


@pytest.mark.parametrize("lens", [[1000, 0, 65, 130], [3000]])
def test_qk_l2norm_chunked_matches_oracle(gdn, lens):
    """use_qk_l2norm on the chunked tensor-core path (the factors 1/|k_t|, 1/|q_t| folded
    into the per-token gate factors; raw bf16 q, k in the products) against the oracle,
    which normalises in fp32."""
    inp = _unnormalised(gdn.workloads.prefill_inputs(lens, seed=43 + len(lens)), seed=7)
    out, ns = gdn.kernel_prefill.run(**to_dev(inp), use_qk_l2norm=True)
    o_ref, s_ref = oracle_prefill(inp, impl=c_oracle, use_qk_l2norm=True)
    assert_match(out, ns, o_ref, s_ref)
    assert gdn._lib.device_error() == 0


def test_qk_l2norm_chunked_equals_serial(gdn):
    inp = to_dev(_unnormalised(gdn.workloads.prefill_inputs([300, 64, 5, 0, 77], seed=44), seed=8))
    o1, s1 = gdn.kernel_prefill.run(**inp, use_qk_l2norm=True)
    o2, s2 = gdn.kernel_prefill.run(**inp, use_qk_l2norm=True, serial=True)
    torch.cuda.synchronize()
    np.testing.assert_allclose(o1.float().cpu().numpy(), o2.float().cpu().numpy(), **OUT_TOL)
    ok, err = state_close(s1.cpu().numpy(), s2.cpu().numpy(), STATE_RTOL)
    assert ok, err
