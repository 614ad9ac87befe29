"""The CPU oracle is pinned against golden vectors produced by the reference's
own Triton kernels (run under the Triton interpreter, ``tests/golden/make_golden.py``).
CPU only."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err, state_close
from oracle import c_oracle
from oracle import gdn_oracle as ref


def _decode_args(g):
    state = ref.bf16_bits_to_f32(g["state"]) if bool(g["has_state"]) else None
    scale = float(g["scale"]) or None
    return (g["q"], g["k"], g["v"], state, g["A_log"], g["a"], g["dt_bias"], g["b"], scale)


def _ulp_diff(x_bits, y_bits):
    x = ref.bf16_bits_to_f32(x_bits)
    y = ref.bf16_bits_to_f32(y_bits)
    return np.max(np.abs(x - y)), np.max(np.abs(y))


@pytest.mark.parametrize("name", ["decode_qk4v8_b3", "decode_qk4v8_b2_nostate"])
@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_decode_oracle_matches_reference_kernel(name, impl):
    g = load_golden(name)
    fn = ref.decode if impl == "numpy" else c_oracle.decode
    out, new_state = fn(*_decode_args(g))
    # bf16 outputs: at most one bf16 rounding step away from the reference's.
    d, m = _ulp_diff(out, g["out_triton"])
    assert d <= 2.0 ** -7 * max(m, 1e-3)
    ok, err = state_close(new_state, g["new_state_triton"], rtol=1e-5)
    assert ok, err


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_prefill_oracle_matches_reference_kernel(impl):
    g = load_golden("prefill_qk4v8_lens1-0-70")
    fn = ref.prefill if impl == "numpy" else c_oracle.prefill
    state = ref.bf16_bits_to_f32(g["state"])
    out, new_state = fn(g["q"], g["k"], g["v"], state, g["A_log"], g["a"], g["dt_bias"], g["b"],
                        g["cu_seqlens"], None)
    d, m = _ulp_diff(out, g["out_triton"])
    assert d <= 2.0 ** -7 * max(m, 1e-3)
    ok, err = state_close(new_state, g["new_state_triton"], rtol=1e-5)
    assert ok, err
    # Empty sequence (index 1): the reference kernel passes the initial state through.
    assert np.array_equal(new_state[1], state[1])


def test_golden_records_torchref_divergence_on_empty_sequence():
    """The definition's torch reference leaves an empty sequence's state at zero,
    the reference kernel copies the initial state; the fixture records both."""
    g = load_golden("prefill_qk4v8_lens1-0-70")
    assert float(g["torchref_empty_seq_state_absmax"]) == 0.0
    assert float(g["torchref_state_maxdiff_nonempty"]) < 1e-5
    assert np.abs(g["new_state_triton"][1]).max() > 0


def test_c_and_numpy_oracles_agree_full_heads(gdn):
    """16 q/k heads, 32 v heads (the benchmark head counts), decode and prefill."""
    wl = gdn.workloads
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    inp = wl.decode_inputs(2, seed=5)
    args = (bits(inp["q"]), bits(inp["k"]), bits(inp["v"]), inp["state"].numpy(),
            inp["A_log"].numpy(), bits(inp["a"]), inp["dt_bias"].numpy(), bits(inp["b"]),
            inp["scale"])
    o1, s1 = ref.decode(*args)
    o2, s2 = c_oracle.decode(*args)
    assert rel_err(ref.bf16_bits_to_f32(o2), ref.bf16_bits_to_f32(o1)) < 1e-2
    assert state_close(s2, s1, rtol=1e-5)[0]

    inp = wl.prefill_inputs([3, 0, 17], seed=6)
    args = (bits(inp["q"]), bits(inp["k"]), bits(inp["v"]), inp["state"].numpy(),
            inp["A_log"].numpy(), bits(inp["a"]), inp["dt_bias"].numpy(), bits(inp["b"]),
            inp["cu_seqlens"].numpy(), inp["scale"])
    o1, s1 = ref.prefill(*args)
    o2, s2 = c_oracle.prefill(*args, nthreads=3)
    assert rel_err(ref.bf16_bits_to_f32(o2), ref.bf16_bits_to_f32(o1)) < 1e-2
    assert state_close(s2, s1, rtol=1e-5)[0]


def test_oracle_l2norm_flag_is_identity_on_unit_vectors(gdn):
    """With q, k already unit-norm (bf16-rounded), the optional normalisation
    changes outputs only at the bf16-rounding level."""
    wl = gdn.workloads
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    inp = wl.decode_inputs(1, seed=7)
    args = (bits(inp["q"]), bits(inp["k"]), bits(inp["v"]), inp["state"].numpy(),
            inp["A_log"].numpy(), bits(inp["a"]), inp["dt_bias"].numpy(), bits(inp["b"]),
            inp["scale"])
    o1, s1 = ref.decode(*args)
    o2, s2 = ref.decode(*args, use_qk_l2norm=True)
    assert rel_err(ref.bf16_bits_to_f32(o2), ref.bf16_bits_to_f32(o1)) < 2e-2
    assert state_close(s2, s1, rtol=2e-2)[0]


def test_pooled_decode_oracle_matches_prefill_per_slot(gdn):
    wl = gdn.workloads
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    B, T, P = 3, 2, 5
    inp = wl.prefill_inputs([T] * B, num_qk_heads=4, num_v_heads=8, seed=8)
    pool = np.random.default_rng(0).normal(0, 0.05, (P, 8, 128, 128)).astype(np.float32)
    idx = np.array([4, -1, 1])
    rs = lambda t: t.reshape(B, T, *t.shape[1:])  # noqa: E731
    out, new_pool = ref.decode_pooled(rs(bits(inp["q"])), rs(bits(inp["k"])), rs(bits(inp["v"])),
                                      pool, idx, inp["A_log"].numpy(), rs(bits(inp["a"])),
                                      inp["dt_bias"].numpy(), rs(bits(inp["b"])), None)
    for i, slot in enumerate(idx):
        if slot < 0:
            assert not out[i].any()
            continue
        sl = slice(i * T, (i + 1) * T)
        o, s = ref.prefill(bits(inp["q"])[sl], bits(inp["k"])[sl], bits(inp["v"])[sl],
                           pool[slot:slot + 1], inp["A_log"].numpy(), bits(inp["a"])[sl],
                           inp["dt_bias"].numpy(), bits(inp["b"])[sl], np.array([0, T]), None)
        assert np.array_equal(out[i], o)
        assert np.array_equal(new_pool[slot], s[0])
    for slot in (0, 2, 3):
        assert np.array_equal(new_pool[slot], pool[slot])


def test_mtp_oracle_matches_flashinfer_reference():
    """Pooled multi-token decode: the oracle against flashinfer's ``_gdn_mtp_reference``
    (the definition-level reference of the serving form; fixture by make_golden.py)."""
    g = load_golden("mtp_qk4v8_b2_t3_pool4")
    pool = ref.bf16_bits_to_f32(g["pool"])
    out, new_pool = ref.decode_pooled(g["q"], g["k"], g["v"], pool, g["indices"], g["A_log"], g["a"],
                                      g["dt_bias"], g["b"], None)
    d, m = _ulp_diff(out, g["out_torchref"])
    assert d <= 2.0 ** -7 * max(m, 1e-3)
    ok, err = state_close(new_pool[g["indices"]], g["final_used_slots_torchref"], rtol=1e-5)
    assert ok, err
    untouched = [s for s in range(pool.shape[0]) if s not in set(g["indices"].tolist())]
    assert all(np.array_equal(new_pool[s], pool[s]) for s in untouched)


# ----------------------------------------------------------------------------- 16 / 32 heads
# BASELINE.json's head counts.  The fixtures keep the reference kernels' outputs and the
# final states of a subset of v-heads; the inputs are regenerated from the seed
# (tests/golden/seeded.py) and checked against the digest the fixture stores.
from golden import seeded  # noqa: E402


def qk16v32_decode_case():
    g = load_golden("decode_qk16v32_b2")
    inp = seeded.decode_qk16v32_inputs(int(g["seed"]))
    assert seeded.digest(*inp) == str(g["inputs_sha256"]), "seeded inputs drifted from the fixture"
    return g, inp


def qk16v32_prefill_case():
    g = load_golden("prefill_qk16v32_lens200-0-65")
    inp = seeded.prefill_qk16v32_inputs([int(x) for x in g["lens"]], int(g["seed"]))
    assert seeded.digest(*inp) == str(g["inputs_sha256"]), "seeded inputs drifted from the fixture"
    return g, inp


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_decode_oracle_matches_reference_kernel_16_32_heads(impl):
    g, (q, k, v, a, b, A_log, dt_bias, state) = qk16v32_decode_case()
    fn = ref.decode if impl == "numpy" else c_oracle.decode
    b16 = seeded.bits
    out, new_state = fn(b16(q), b16(k), b16(v), state.numpy(), A_log.numpy(), b16(a), dt_bias.numpy(), b16(b), None)
    d, m = _ulp_diff(out, g["out_triton"])
    assert d <= 2.0 ** -7 * max(m, 1e-3)
    ok, err = state_close(new_state[:, g["stored_heads"]], g["new_state_triton"], rtol=1e-5)
    assert ok, err


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_prefill_oracle_matches_reference_kernel_16_32_heads(impl):
    g, (q, k, v, a, b, A_log, dt_bias, state, cu) = qk16v32_prefill_case()
    fn = ref.prefill if impl == "numpy" else c_oracle.prefill
    b16 = seeded.bits
    out, new_state = fn(b16(q), b16(k), b16(v), state.numpy(), A_log.numpy(), b16(a), dt_bias.numpy(), b16(b),
                        cu.numpy(), None)
    d, m = _ulp_diff(out, g["out_triton"])
    assert d <= 2.0 ** -7 * max(m, 1e-3)
    ok, err = state_close(new_state[:, g["stored_heads"]], g["new_state_triton"], rtol=1e-5)
    assert ok, err
    assert bool(g["empty_seq_passthrough"]) and np.array_equal(new_state[1], state[1].numpy())
