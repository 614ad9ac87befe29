"""Decode parity on the GPU: the CUDA path (through the C ABI) against the
golden vectors of the reference kernel and against the CPU oracle.

Tolerances (as the specification states them): bf16 output atol = rtol = 1e-2;
fp32 final state within 1e-3 relative (per (sequence, head): max-abs error and
Frobenius error, each relative to the reference state's max-abs / norm)."""
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


def oracle_decode(inp, **kw):
    st = inp["state"]
    return ref.decode(bits(inp["q"]), bits(inp["k"]), bits(inp["v"]),
                      None if st is None else st.cpu().numpy(), inp["A_log"].cpu().numpy(),
                      bits(inp["a"]), inp["dt_bias"].cpu().numpy(), bits(inp["b"]), inp["scale"], **kw)


def assert_match(out, new_state, o_ref_bits, s_ref):
    o = out.float().cpu().numpy()
    o_ref = ref.bf16_bits_to_f32(o_ref_bits)
    np.testing.assert_allclose(o, o_ref, **OUT_TOL)
    ok, err = state_close(new_state.cpu().numpy(), s_ref, STATE_RTOL)
    assert ok, f"state rel err {err}"


@pytest.mark.parametrize("name", ["decode_qk4v8_b3", "decode_qk4v8_b2_nostate"])
def test_golden_reference_kernel(gdn, name):
    g = load_golden(name)
    dev = "cuda"
    tb = lambda x: torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev)  # noqa: E731
    state = torch.from_numpy(ref.bf16_bits_to_f32(g["state"])).to(dev) if bool(g["has_state"]) else None
    out, ns = gdn.kernel_decode.run(tb(g["q"]), tb(g["k"]), tb(g["v"]), state,
                                    torch.from_numpy(g["A_log"]).to(dev), tb(g["a"]),
                                    torch.from_numpy(g["dt_bias"]).to(dev), tb(g["b"]),
                                    float(g["scale"]) or None)
    torch.cuda.synchronize()
    assert out.shape == (g["q"].shape[0], 1, g["v"].shape[2], 128) and out.dtype == torch.bfloat16
    assert_match(out, ns, g["out_triton"], g["new_state_triton"])


@pytest.mark.parametrize("B", [1, 3, 17, 64])
def test_random_full_heads(gdn, B):
    inp = gdn.workloads.decode_inputs(B, seed=100 + B)
    out, ns = gdn.kernel_decode.run(**to_dev(inp))
    o_ref, s_ref = oracle_decode(inp)
    assert_match(out, ns, o_ref, s_ref)
    assert gdn._lib.device_error() == 0


def test_zero_state_and_default_scale(gdn):
    inp = gdn.workloads.decode_inputs(5, seed=7)
    inp["state"] = None
    for scale in (None, 0.0):
        inp["scale"] = scale
        out, ns = gdn.kernel_decode.run(**to_dev(inp))
        o_ref, s_ref = oracle_decode(inp)
        assert_match(out, ns, o_ref, s_ref)


def test_custom_scale_and_gva_ratio_4(gdn):
    inp = gdn.workloads.decode_inputs(6, num_qk_heads=8, num_v_heads=32, seed=8)
    inp["scale"] = 0.3
    out, ns = gdn.kernel_decode.run(**to_dev(inp))
    o_ref, s_ref = oracle_decode(inp)
    assert_match(out, ns, o_ref, s_ref)


def test_qk_l2norm_flag(gdn):
    inp = gdn.workloads.decode_inputs(4, seed=9)
    # un-normalised q/k so the flag matters
    inp["q"] = (inp["q"].float() * 3.0).bfloat16()
    inp["k"] = (inp["k"].float() * 0.5).bfloat16()
    out, ns = gdn.kernel_decode.run(**to_dev(inp), use_qk_l2norm=True)
    o_ref, s_ref = oracle_decode(inp, use_qk_l2norm=True)
    assert_match(out, ns, o_ref, s_ref)


def test_in_place_state_update(gdn):
    inp = gdn.workloads.decode_inputs(8, seed=10)
    d = to_dev(inp)
    st = d["state"].clone()
    out = torch.empty(8, 1, 32, 128, dtype=torch.bfloat16, device="cuda")
    gdn.kernel_decode.run_dps(d["q"], d["k"], d["v"], st, d["A_log"], d["a"], d["dt_bias"], d["b"],
                              d["scale"], out, st)
    o_ref, s_ref = oracle_decode(inp)
    assert_match(out, st, o_ref, s_ref)


def test_strided_qkv_views(gdn):
    """q, k, v as views into one fused projection buffer (batch stride != dense)."""
    B, HQ, HV, D = 4, 16, 32, 128
    inp = gdn.workloads.decode_inputs(B, seed=11)
    fused = torch.zeros(B, 1, (2 * HQ + HV) * D + 64, dtype=torch.bfloat16)
    fused[..., :HQ * D] = inp["q"].reshape(B, 1, -1)
    fused[..., HQ * D:2 * HQ * D] = inp["k"].reshape(B, 1, -1)
    fused[..., 2 * HQ * D:(2 * HQ + HV) * D] = inp["v"].reshape(B, 1, -1)
    fd = fused.cuda()
    q = fd[..., :HQ * D].unflatten(-1, (HQ, D))
    k = fd[..., HQ * D:2 * HQ * D].unflatten(-1, (HQ, D))
    v = fd[..., 2 * HQ * D:(2 * HQ + HV) * D].unflatten(-1, (HV, D))
    assert not q.is_contiguous()
    d = to_dev(inp)
    out, ns = gdn.kernel_decode.run(q, k, v, d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"], None)
    o_ref, s_ref = oracle_decode(inp)
    assert_match(out, ns, o_ref, s_ref)


def test_full_size_b1024_subset_and_batch_invariance(gdn):
    """configs[2] size on one GPU: every sequence is independent, so a sample of
    sequences is checked against the oracle and against single-sequence calls."""
    inp = gdn.workloads.decode_inputs(1024, seed=12, device="cuda")
    out, ns = gdn.kernel_decode.run(**inp)
    torch.cuda.synchronize()
    rng = np.random.default_rng(0)
    for i in sorted(rng.choice(1024, 6, replace=False).tolist()):
        sub = {k: (v[i:i + 1] if torch.is_tensor(v) and v.shape[0] == 1024 else v) for k, v in inp.items()}
        o1, s1 = gdn.kernel_decode.run(**sub)
        assert torch.equal(o1, out[i:i + 1]) and torch.equal(s1, ns[i:i + 1])
        cpu = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in sub.items()}
        o_ref, s_ref = c_oracle.decode(bits(cpu["q"]), bits(cpu["k"]), bits(cpu["v"]), cpu["state"].numpy(),
                                       cpu["A_log"].numpy(), bits(cpu["a"]), cpu["dt_bias"].numpy(),
                                       bits(cpu["b"]), cpu["scale"])
        assert_match(out[i:i + 1], ns[i:i + 1], o_ref, s_ref)


def test_decode_chain_equals_prefill_recurrence(gdn):
    """T successive decode steps equal one T-token prefill of the oracle."""
    T, HQ, HV = 9, 16, 32
    inp = gdn.workloads.prefill_inputs([T], seed=13)
    d = to_dev(inp)
    st = d["state"]
    outs = []
    for t in range(T):
        o, st = gdn.kernel_decode.run(d["q"][t:t + 1, None], d["k"][t:t + 1, None], d["v"][t:t + 1, None],
                                      st, d["A_log"], d["a"][t:t + 1, None], d["dt_bias"],
                                      d["b"][t:t + 1, None], None)
        outs.append(o[:, 0])
    out = torch.cat(outs)
    o_ref, s_ref = ref.prefill(bits(inp["q"]), bits(inp["k"]), bits(inp["v"]), inp["state"].numpy(),
                               inp["A_log"].numpy(), bits(inp["a"]), inp["dt_bias"].numpy(),
                               bits(inp["b"]), inp["cu_seqlens"].numpy(), None)
    assert_match(out, st, o_ref, s_ref)


def test_invalid_arguments_raise_before_launch(gdn):
    inp = to_dev(gdn.workloads.decode_inputs(2, seed=14))
    bad = dict(inp)
    bad["q"] = inp["q"].float()
    with pytest.raises(TypeError):
        gdn.kernel_decode.run(**bad)
    out = torch.empty(2, 1, 32, 128, dtype=torch.bfloat16, device="cuda")
    ns = inp["state"][:, :, :, :].clone()
    overlap = torch.empty(2 * 32 * 128 * 128 + 4, device="cuda")
    with pytest.raises(gdn._lib.GDNError, match="overlap"):
        gdn.kernel_decode.run_dps(inp["q"], inp["k"], inp["v"], overlap[:-4].view(2, 32, 128, 128),
                                  inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], None, out,
                                  overlap[4:].view(2, 32, 128, 128))
    del ns


def test_golden_reference_kernel_16_32_heads(gdn):
    """BASELINE.json's head counts (16 q/k, 32 v heads) against the reference kernel."""
    from test_oracle import qk16v32_decode_case

    g, (q, k, v, a, b, A_log, dt_bias, state) = qk16v32_decode_case()
    dev = lambda t: t.cuda()  # noqa: E731
    out, ns = gdn.kernel_decode.run(dev(q), dev(k), dev(v), dev(state), dev(A_log), dev(a), dev(dt_bias), dev(b),
                                    None)
    torch.cuda.synchronize()
    assert_match(out, ns[:, torch.from_numpy(g["stored_heads"]).cuda()], g["out_triton"], g["new_state_triton"])
