"""Pooled multi-token decode (``kernel_mtp``, C ABI ``gdn_decode_pooled``) on the GPU
against flashinfer's ``_gdn_mtp_reference`` fixture and the CPU oracle.
Tolerances as everywhere: bf16 outputs atol = rtol = 1e-2, states 1e-3 relative."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden, state_close
from oracle import gdn_oracle as ref

pytestmark = pytest.mark.gpu
OUT_TOL = dict(atol=1e-2, rtol=1e-2)


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def mtp_inputs(gdn, B, T, P, HQ=16, HV=32, seed=0):
    """B sequences x T tokens in the BASELINE distributions, a pool of P states."""
    wl = gdn.workloads
    inp = wl.prefill_inputs([T] * B, num_qk_heads=HQ, num_v_heads=HV, seed=seed)
    rs = lambda t: t.reshape(B, T, *t.shape[1:])  # noqa: E731
    gen = torch.Generator().manual_seed(seed + 1)
    pool = torch.randn(P, HV, 128, 128, generator=gen) * 0.05
    return dict(q=rs(inp["q"]), k=rs(inp["k"]), v=rs(inp["v"]), a=rs(inp["a"]), b=rs(inp["b"]),
                A_log=inp["A_log"], dt_bias=inp["dt_bias"], pool=pool)


def oracle(d, idx, **kw):
    return ref.decode_pooled(bits(d["q"]), bits(d["k"]), bits(d["v"]), d["pool"].numpy(), np.asarray(idx),
                             d["A_log"].numpy(), bits(d["a"]), d["dt_bias"].numpy(), bits(d["b"]), None, **kw)


def run_gpu(gdn, d, idx, inter=None, **kw):
    c = {k: v.cuda() for k, v in d.items()}
    return gdn.kernel_mtp.run(c["q"], c["k"], c["v"], c["pool"], torch.tensor(idx, device="cuda"), c["A_log"],
                              c["a"], c["dt_bias"], c["b"], None, inter, **kw)


def check(out, pool, o_ref, p_ref):
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.bf16_bits_to_f32(o_ref), **OUT_TOL)
    ok, err = state_close(pool.cpu().numpy(), p_ref, 1e-3)
    assert ok, f"state rel err {err}"


def test_golden_flashinfer_mtp_reference(gdn):
    g = load_golden("mtp_qk4v8_b2_t3_pool4")
    tb = lambda x: torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()  # noqa: E731
    pool = torch.from_numpy(ref.bf16_bits_to_f32(g["pool"])).cuda()
    idx = torch.from_numpy(g["indices"]).cuda()
    out, fin = gdn.kernel_mtp.run(tb(g["q"]), tb(g["k"]), tb(g["v"]), pool, idx, torch.from_numpy(g["A_log"]).cuda(),
                                  tb(g["a"]), torch.from_numpy(g["dt_bias"]).cuda(), tb(g["b"]), None)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.bf16_bits_to_f32(g["out_torchref"]), **OUT_TOL)
    ok, err = state_close(fin[idx.long()].cpu().numpy(), g["final_used_slots_torchref"], 1e-3)
    assert ok, err
    assert torch.equal(fin[0], pool[0]) and torch.equal(fin[2], pool[2])  # untouched slots


@pytest.mark.parametrize("T", [1, 4, 8, 19])  # 1: single-token kernel; 4, 8: chunked; 19: general kernel, two token groups
def test_random_pool_with_padding_entry(gdn, T):
    d = mtp_inputs(gdn, B=5, T=T, P=8, seed=200 + T)
    idx = [6, -1, 0, 3, 7]
    out, fin = run_gpu(gdn, d, idx)
    torch.cuda.synchronize()
    o_ref, p_ref = oracle(d, idx)
    check(out, fin, o_ref, p_ref)
    assert not out[1].float().abs().any()  # the padded entry's outputs are zero
    assert gdn._lib.device_error() == 0


def test_many_items_per_warp(gdn):
    """160 sequences = 81,920 eight-row items, several per warp of the persistent
    grid, so every warp cycles both stages of its copy pipeline; padded entries
    interleaved."""
    B, T, P = 160, 2, 170
    d = mtp_inputs(gdn, B=B, T=T, P=P, HQ=16, HV=32, seed=215)
    idx = list(np.random.default_rng(215).permutation(P)[:B])
    idx[7] = idx[100] = -1
    out, fin = run_gpu(gdn, d, idx)
    torch.cuda.synchronize()
    o_ref, p_ref = oracle(d, idx)
    check(out, fin, o_ref, p_ref)
    assert gdn._lib.device_error() == 0


@pytest.mark.parametrize("T", [3, 8])
def test_rows_on_8_byte_boundaries(gdn, T):
    """q/k/v rows 8-byte but not 16-byte aligned (head stride 132 elements): the
    general kernel runs instead of the bulk-copy pipeline, same results."""
    B, P = 4, 6
    d = mtp_inputs(gdn, B=B, T=T, P=P, seed=216 + T)
    idx = [5, 0, -1, 2]
    o_ref, p_ref = oracle(d, idx)
    c = {k: v.cuda() for k, v in d.items()}

    def pad(x):  # same values, rows starting 4 elements (8 bytes) into a 132-wide buffer
        big = torch.zeros(*x.shape[:-1], 132, dtype=x.dtype, device=x.device)
        big[..., 4:] = x
        return big[..., 4:]

    q, k, v = pad(c["q"]), pad(c["k"]), pad(c["v"])
    assert q.stride(2) == 132 and q.data_ptr() % 16 == 8
    out, fin = gdn.kernel_mtp.run(q, k, v, c["pool"], torch.tensor(idx, device="cuda"), c["A_log"], c["a"],
                                  c["dt_bias"], c["b"], None)
    torch.cuda.synchronize()
    check(out, fin, o_ref, p_ref)


def test_intermediate_states_and_in_place_pool(gdn):
    B, T, P = 3, 5, 4
    d = mtp_inputs(gdn, B=B, T=T, P=P, seed=210)
    idx = [2, 0, 3]
    o_ref, p_ref, inter_ref = oracle(d, idx, return_intermediate=True)
    c = {k: v.cuda() for k, v in d.items()}
    pool = c["pool"].clone()
    inter = torch.full((P, T, 32, 128, 128), float("nan"), device="cuda")
    out = torch.empty(B, T, 32, 128, dtype=torch.bfloat16, device="cuda")
    gdn.kernel_mtp.run_dps(c["q"], c["k"], c["v"], pool, torch.tensor(idx, device="cuda"), c["A_log"], c["a"],
                           c["dt_bias"], c["b"], None, out, pool, inter)  # in place: final_state is the pool
    torch.cuda.synchronize()
    check(out, pool, o_ref, p_ref)
    for (slot, t), s_ref in inter_ref.items():
        ok, err = state_close(inter[slot, t].cpu().numpy()[None], s_ref[None], 1e-3)
        assert ok, (slot, t, err)
    assert torch.isnan(inter[1]).all()  # slot 1 is not named: its buffer is not written


def test_qk_l2norm_and_gva_ratio_4(gdn):
    d = mtp_inputs(gdn, B=2, T=3, P=3, HQ=8, HV=32, seed=220)
    d["q"] = (d["q"].float() * 2.0).bfloat16()
    idx = [1, 2]
    out, fin = run_gpu(gdn, d, idx, use_qk_l2norm=True)
    torch.cuda.synchronize()
    o_ref, p_ref = oracle(d, idx, use_qk_l2norm=True)
    check(out, fin, o_ref, p_ref)


def test_one_token_equals_dense_decode(gdn):
    """T = 1 with indices 0..B-1 is the single-token decode of the dense state batch,
    up to fp32 rounding: the pooled kernel reduces over 8 lanes per row and takes
    S.k on the undecayed row (g (S.k) instead of (g S).k), the dense one over 32
    lanes on the decayed row.  States agree to 1e-6 absolute (entries ~0.05),
    outputs to one bf16 ulp."""
    B = 6
    inp = gdn.workloads.decode_inputs(B, seed=230)
    c = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}
    o1, s1 = gdn.kernel_decode.run(**c)
    o2, s2 = gdn.kernel_mtp.run(c["q"], c["k"], c["v"], c["state"], torch.arange(B, device="cuda"), c["A_log"],
                                c["a"], c["dt_bias"], c["b"], c["scale"])
    torch.cuda.synchronize()
    torch.testing.assert_close(s2, s1, atol=1e-6, rtol=0)
    torch.testing.assert_close(o2.float(), o1.float(), atol=1e-3, rtol=2 ** -7)


def test_index_beyond_pool_sets_device_error(gdn):
    d = mtp_inputs(gdn, B=2, T=2, P=2, seed=240)
    gdn._lib.device_error(clear=True)
    out, fin = run_gpu(gdn, d, [0, 5])
    torch.cuda.synchronize()
    assert gdn._lib.device_error(clear=True) & gdn._lib.GDN_DEVERR_BAD_INDEX
    assert not out[1].float().abs().any()


@pytest.mark.parametrize("T,l2", [(2, False), (2, True), (3, True), (4, False), (4, True), (5, False), (6, True), (7, False), (8, False), (8, True)])
def test_chunked_tokens_match_token_serial_kernel(gdn, T, l2):
    """2 to 8 tokens without intermediate states run the chunked kernel (every token's
    products with the state from the item's initial rows, the token recurrence on
    scalars through the Gram matrix of q and k); a call that also asks for the
    intermediate states runs the token-serial kernel.  Both must give the same outputs
    and final states on the same inputs, within fp32 rounding."""
    B, P = 37, 40  # 37 x 32 x 16 items: several per warp, padded entries among them
    d = mtp_inputs(gdn, B=B, T=T, P=P, seed=250 + T)
    if l2:
        d["q"] = (d["q"].float() * 3.0).bfloat16()
        d["k"] = (d["k"].float() * 0.5).bfloat16()
    idx = list(np.random.default_rng(250 + T).permutation(P)[:B])
    idx[3] = idx[20] = -1
    c = {k: v.cuda() for k, v in d.items()}
    ix = torch.tensor(idx, device="cuda")
    out1, fin1 = gdn.kernel_mtp.run(c["q"], c["k"], c["v"], c["pool"], ix, c["A_log"], c["a"], c["dt_bias"],
                                    c["b"], None, use_qk_l2norm=l2)
    inter = torch.empty(P, T, 32, 128, 128, device="cuda")
    out2, fin2 = gdn.kernel_mtp.run(c["q"], c["k"], c["v"], c["pool"], ix, c["A_log"], c["a"], c["dt_bias"],
                                    c["b"], None, inter, use_qk_l2norm=l2)
    torch.cuda.synchronize()
    torch.testing.assert_close(fin1, fin2, atol=2e-6, rtol=1e-5)
    torch.testing.assert_close(out1.float(), out2.float(), atol=1e-3, rtol=2 ** -7)
    assert torch.equal(fin1[[i for i in range(P) if i not in idx]], c["pool"][[i for i in range(P) if i not in idx]])
    assert not out1[3].float().abs().any() and not out1[20].float().abs().any()
    o_ref, p_ref = oracle(d, idx, use_qk_l2norm=l2)
    check(out1, fin1, o_ref, p_ref)
    assert gdn._lib.device_error() == 0


@pytest.mark.parametrize("T", [3, 4])
def test_fused_projection_views(gdn, T):
    """q, k, v as views of one fused projection buffer [B, T, HQ + HQ + HV + 8, 128] (every
    batch, token and head stride differs from a contiguous tensor; rows stay 16-byte aligned):
    same results as contiguous copies."""
    B, P, HQ, HV = 6, 9, 16, 32
    d = mtp_inputs(gdn, B=B, T=T, P=P, seed=260 + T)
    idx = [4, -1, 0, 8, 2, 6]
    c = {k: v.cuda() for k, v in d.items()}
    buf = torch.zeros(B, T, 2 * HQ + HV + 8, 128, dtype=torch.bfloat16, device="cuda")
    buf[:, :, :HQ] = c["q"]
    buf[:, :, HQ:2 * HQ] = c["k"]
    buf[:, :, 2 * HQ:2 * HQ + HV] = c["v"]
    q, k, v = buf[:, :, :HQ], buf[:, :, HQ:2 * HQ], buf[:, :, 2 * HQ:2 * HQ + HV]
    assert not q.is_contiguous() and q.stride(1) == (2 * HQ + HV + 8) * 128
    ix = torch.tensor(idx, device="cuda")
    o1, f1 = gdn.kernel_mtp.run(q, k, v, c["pool"], ix, c["A_log"], c["a"], c["dt_bias"], c["b"], None)
    o2, f2 = gdn.kernel_mtp.run(c["q"], c["k"], c["v"], c["pool"], ix, c["A_log"], c["a"], c["dt_bias"], c["b"],
                                None)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(f1, f2)
    o_ref, p_ref = oracle(d, idx)
    check(o1, f1, o_ref, p_ref)


def test_one_token_in_place_padding_and_bad_index(gdn):
    """One token without intermediate states runs the single-token decode kernel on the
    indexed slots: in place (the pool is its own output), a padded entry leaves zeros and
    touches no slot, an index beyond the pool raises GDN_DEVERR_BAD_INDEX."""
    B, P = 5, 7
    d = mtp_inputs(gdn, B=B, T=1, P=P, seed=270)
    idx = [6, -1, 0, 3, 1]
    c = {k: v.cuda() for k, v in d.items()}
    pool = c["pool"].clone()
    out = torch.empty(B, 1, 32, 128, dtype=torch.bfloat16, device="cuda")
    gdn._lib.device_error(clear=True)
    gdn.kernel_mtp.run_dps(c["q"], c["k"], c["v"], pool, torch.tensor(idx, device="cuda", dtype=torch.int32),
                           c["A_log"], c["a"], c["dt_bias"], c["b"], None, out, pool)
    torch.cuda.synchronize()
    o_ref, p_ref = oracle(d, idx)
    check(out, pool, o_ref, p_ref)
    assert not out[1].float().abs().any()
    assert torch.equal(pool[[2, 4, 5]], c["pool"][[2, 4, 5]])  # slots no entry names
    assert gdn._lib.device_error(clear=True) == 0
    out2, _ = run_gpu(gdn, d, [0, 9, 2, 3, 4])
    torch.cuda.synchronize()
    assert gdn._lib.device_error(clear=True) & gdn._lib.GDN_DEVERR_BAD_INDEX
    assert not out2[1].float().abs().any()
