"""Generate the golden fixtures in this directory from the reference itself.

Runs the reference solution's own Triton kernels
(``solution/triton/kernel_decode.py::run`` and ``kernel_prefill.py::run``) on
the CPU under ``TRITON_INTERPRET=1``, plus the definition's torch reference
recurrence shipped with ``flashinfer==0.6.11.post2``
(``flashinfer/trace/templates/gdn.py``: ``_gdn_decode_reference``,
``_gdn_prefill_reference``, and ``_gdn_mtp_reference`` for the pooled
multi-token decode, which the kit itself does not have), on small seeded inputs, and stores inputs and
outputs as compressed ``.npz`` files (the torch reference's states are kept
only as their max difference from the Triton kernels' states, to keep the
fixtures small).  bf16 tensors are stored as uint16 bit
patterns; the initial states are drawn as bf16-representable fp32 values so
they can be stored as uint16 too.

Usage (needs the reference checkout; not run by the tests):
    python tests/golden/make_golden.py /path/to/reference [qk16v32]
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from seeded import (STORED_HEADS, bits, decode_qk16v32_inputs, digest, make_inputs,  # noqa: E402
                    prefill_qk16v32_inputs)


def main(ref_root: str, only: str | None = None) -> None:
    sys.path.insert(0, str(Path(ref_root) / "solution" / "triton"))
    import kernel_decode  # reference decode entry point
    import kernel_prefill  # reference prefill entry point
    from flashinfer.trace.templates.gdn import _gdn_decode_reference, _gdn_mtp_reference, _gdn_prefill_reference

    if only in (None, "qk16v32"):
        make_qk16v32(kernel_decode, kernel_prefill, _gdn_decode_reference, _gdn_prefill_reference)
    if only == "qk16v32":
        return

    # ---- decode, the reference definition's own head counts (qk4 / v8) ----
    cases = [("decode_qk4v8_b3", 3, 4, 8, 11, True, None),
             ("decode_qk4v8_b2_nostate", 2, 4, 8, 12, False, 0.25)]
    for name, B, HQ, HV, seed, with_state, scale in cases:
        q, k, v, a, b, A_log, dt_bias, state = make_inputs(
            (B, 1, HQ, 128), (B, 1, HV, 128), (B, 1, HV), (B, HV, 128, 128), seed)
        st = state if with_state else None
        o_tr, s_tr = kernel_decode.run(q, k, v, st, A_log, a, dt_bias, b, scale)
        o_fi, s_fi = _gdn_decode_reference(q, k, v, st, A_log, a, dt_bias, b, scale)
        np.savez_compressed(
            HERE / f"{name}.npz", q=bits(q), k=bits(k), v=bits(v), a=bits(a), b=bits(b),
            A_log=A_log.numpy(), dt_bias=dt_bias.numpy(),
            state=bits(state.bfloat16()) if with_state else np.zeros(0, np.uint16),
            has_state=np.array(with_state), scale=np.float32(0.0 if scale is None else scale),
            out_triton=bits(o_tr), new_state_triton=s_tr.numpy(),
            out_torchref=bits(o_fi),
            torchref_state_maxdiff=np.float32((s_tr - s_fi).abs().max().item()))
        print(name, "triton vs torch-ref: out", (o_tr.float() - o_fi.float()).abs().max().item(),
              "state", (s_tr - s_fi).abs().max().item())

    # ---- prefill: an empty sequence, a 1-token one, and one crossing the 64-token chunk ----
    lens = [1, 0, 70]
    HQ, HV = 4, 8
    T, N = sum(lens), len(lens)
    q, k, v, a, b, A_log, dt_bias, state = make_inputs(
        (T, HQ, 128), (T, HV, 128), (T, HV), (N, HV, 128, 128), 21)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    o_tr, s_tr = kernel_prefill.run(q, k, v, state, A_log, a, dt_bias, b, cu, None)
    o_fi, s_fi = _gdn_prefill_reference(q, k, v, state, A_log, a, dt_bias, b, cu, None)
    np.savez_compressed(
        HERE / "prefill_qk4v8_lens1-0-70.npz", q=bits(q), k=bits(k), v=bits(v), a=bits(a),
        b=bits(b), A_log=A_log.numpy(), dt_bias=dt_bias.numpy(), state=bits(state.bfloat16()),
        cu_seqlens=cu.numpy(), out_triton=bits(o_tr), new_state_triton=s_tr.numpy(),
        out_torchref=bits(o_fi),
        torchref_state_maxdiff_nonempty=np.float32(
            max((s_tr[i] - s_fi[i]).abs().max().item() for i in (0, 2))),
        torchref_empty_seq_state_absmax=np.float32(s_fi[1].abs().max().item()))
    print("prefill triton vs torch-ref: out", (o_tr.float() - o_fi.float()).abs().max().item(),
          "state (non-empty seqs)", max((s_tr[i] - s_fi[i]).abs().max().item() for i in (0, 2)),
          "empty-seq state: triton passes through", (s_tr[1] - state[1]).abs().max().item(),
          "torch-ref writes zeros", s_fi[1].abs().max().item())

    # ---- multi-token decode against a state pool (flashinfer's _gdn_mtp_reference; the
    #      reference kit has no multi-token entry point): 2 sequences x 3 tokens, pool of 4 ----
    B, T, P, HQ, HV = 2, 3, 4, 4, 8
    q, k, v, a, b, A_log, dt_bias, _ = make_inputs((B, T, HQ, 128), (B, T, HV, 128), (B, T, HV), (1, 1, 1, 1), 31)
    gen = torch.Generator()
    gen.manual_seed(32)
    pool = (torch.randn(P, HV, 128, 128, generator=gen) * 0.05).bfloat16().float()
    idx = torch.tensor([3, 1], dtype=torch.int32)
    o_fi, pool_fi = _gdn_mtp_reference(q, k, v, pool, idx, A_log, a, dt_bias, b, None)
    np.savez_compressed(
        HERE / "mtp_qk4v8_b2_t3_pool4.npz", q=bits(q), k=bits(k), v=bits(v), a=bits(a), b=bits(b),
        A_log=A_log.numpy(), dt_bias=dt_bias.numpy(), pool=bits(pool.bfloat16()), indices=idx.numpy(),
        out_torchref=bits(o_fi), final_used_slots_torchref=pool_fi[idx.long()].numpy())
    print("mtp: pool slots", idx.tolist(), "untouched slots unchanged:",
          bool(torch.equal(pool_fi[0], pool[0]) and torch.equal(pool_fi[2], pool[2])))


def make_qk16v32(kernel_decode, kernel_prefill, decode_ref, prefill_ref) -> None:
    """BASELINE.json's head counts (16 q/k heads, 32 v heads; the reference kernels hard-code
    the GVA ratio 2, which these keep).  Inputs are regenerated from the seed by the tests
    (``seeded.py``; the fixture keeps their digest); stored: every output and the final
    states of the v-heads in ``STORED_HEADS``."""
    heads = torch.tensor(STORED_HEADS)
    q, k, v, a, b, A_log, dt_bias, state = decode_qk16v32_inputs()
    o_tr, s_tr = kernel_decode.run(q, k, v, state, A_log, a, dt_bias, b, None)
    o_fi, s_fi = decode_ref(q, k, v, state, A_log, a, dt_bias, b, None)
    np.savez_compressed(
        HERE / "decode_qk16v32_b2.npz", seed=np.int64(13), stored_heads=heads.numpy(),
        inputs_sha256=np.array(digest(q, k, v, a, b, A_log, dt_bias, state)),
        out_triton=bits(o_tr), new_state_triton=s_tr[:, heads].numpy(),
        torchref_out_maxdiff=np.float32((o_tr.float() - o_fi.float()).abs().max().item()),
        torchref_state_maxdiff=np.float32((s_tr - s_fi).abs().max().item()))
    print("decode qk16v32 triton vs torch-ref: out", (o_tr.float() - o_fi.float()).abs().max().item(),
          "state", (s_tr - s_fi).abs().max().item())

    lens = [200, 0, 65]  # 4 chunks (3 full + 8 tokens), an empty sequence, 2 chunks (1 full + 1 token)
    q, k, v, a, b, A_log, dt_bias, state, cu = prefill_qk16v32_inputs(lens)
    o_tr, s_tr = kernel_prefill.run(q, k, v, state, A_log, a, dt_bias, b, cu, None)
    o_fi, s_fi = prefill_ref(q, k, v, state, A_log, a, dt_bias, b, cu, None)
    np.savez_compressed(
        HERE / "prefill_qk16v32_lens200-0-65.npz", seed=np.int64(22), lens=np.array(lens),
        stored_heads=heads.numpy(), inputs_sha256=np.array(digest(q, k, v, a, b, A_log, dt_bias, state, cu)),
        out_triton=bits(o_tr), new_state_triton=s_tr[:, heads].numpy(),
        torchref_out_maxdiff=np.float32((o_tr.float() - o_fi.float()).abs().max().item()),
        torchref_state_maxdiff_nonempty=np.float32(
            max((s_tr[i] - s_fi[i]).abs().max().item() for i in (0, 2))),
        empty_seq_passthrough=np.array(bool(torch.equal(s_tr[1], state[1]))))
    print("prefill qk16v32 triton vs torch-ref: out", (o_tr.float() - o_fi.float()).abs().max().item(),
          "state (non-empty seqs)", max((s_tr[i] - s_fi[i]).abs().max().item() for i in (0, 2)))


if __name__ == "__main__":
    if len(sys.argv) not in (2, 3):
        sys.exit("usage: make_golden.py <reference checkout> [qk16v32]")
    main(sys.argv[1], sys.argv[2] if len(sys.argv) == 3 else None)
