"""Harness shim (``harness``): flashinfer-bench workload records (definition + safetensors
blobs, the schema of the reference's recorded traces) loaded and run through the drop-in
``run``s.  The contest dataset is not available offline, so a dataset of the same shape
is written here: qk4/v8 decode and prefill workloads (the reference's definitions),
a workload without a state, a duplicate record in a trace file and a foreign definition.
GPU results are checked against the CPU oracle (bf16 outputs atol = rtol = 1e-2, states
1e-3 relative)."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch
from safetensors.torch import save_file

from conftest import state_close
from oracle import gdn_oracle as ref

DEC = "gdn_decode_qk4_v8_d128_k_last"
PRE = "gdn_prefill_qk4_v8_d128_k_last"


def _record(definition, uuid, tensors, root, axes, scale):
    rel = f"./blob/workloads/gdn/{definition}/{definition}_{uuid}.safetensors"
    path = root / rel
    path.parent.mkdir(parents=True, exist_ok=True)
    save_file({k: v.contiguous() for k, v in tensors.items()}, str(path))
    inputs = {k: {"type": "safetensors", "path": rel, "tensor_key": k} for k in tensors}
    inputs["scale"] = {"type": "scalar", "value": scale}
    return {"definition": definition, "workload": {"axes": axes, "inputs": inputs, "uuid": uuid}}


@pytest.fixture()
def dataset(gdn, tmp_path):
    wl = gdn.workloads
    d = wl.decode_inputs(2, num_qk_heads=4, num_v_heads=8, seed=400)
    keys = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")
    r1 = _record(DEC, "dec-0001", {k: d[k] for k in keys}, tmp_path, {"batch_size": 2}, d["scale"])
    d2 = wl.decode_inputs(1, num_qk_heads=4, num_v_heads=8, seed=401)
    r2 = _record(DEC, "dec-0002", {k: d2[k] for k in keys if k != "state"}, tmp_path, {"batch_size": 1},
                 d2["scale"])
    p = wl.prefill_inputs([5, 70], num_qk_heads=4, num_v_heads=8, seed=402)
    r3 = _record(PRE, "pre-0001", {k: p[k] for k in keys + ("cu_seqlens",)}, tmp_path,
                 {"total_seq_len": 75, "num_seqs": 2, "len_cu_seqlens": 3}, p["scale"])
    (tmp_path / "workloads").mkdir()
    with open(tmp_path / "workloads" / "gdn.jsonl", "w") as f:
        for r in (r1, r2, r3):
            f.write(json.dumps(r) + "\n")
        f.write(json.dumps({"definition": "rmsnorm_h4096", "workload": {"inputs": {}, "uuid": "x"}}) + "\n")
    with open(tmp_path / "traces.jsonl", "w") as f:  # a trace line repeats a workload
        f.write(json.dumps({**r1, "solution": "s", "evaluation": {"status": "PASSED"}}) + "\n\n")
    return tmp_path, {"dec-0001": d, "dec-0002": d2, "pre-0001": p}


def test_find_and_load_records(gdn, dataset):
    root, src = dataset
    h = gdn.harness
    recs = h.find_records(root)
    assert sorted(r["workload"]["uuid"] for r in recs) == ["dec-0001", "dec-0002", "pre-0001"]
    assert [r["workload"]["uuid"] for r in h.find_records(root, PRE)] == ["pre-0001"]
    assert h.kind_of(DEC) == "decode" and h.kind_of(PRE) == "prefill"
    with pytest.raises(ValueError):
        h.kind_of("rmsnorm_h4096")
    by = {r["workload"]["uuid"]: r for r in recs}
    kw = h.load_inputs(by["pre-0001"], root, device="cpu")
    assert list(kw) == ["q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens", "scale"]
    assert torch.equal(kw["q"], src["pre-0001"]["q"]) and kw["q"].dtype == torch.bfloat16
    assert torch.equal(kw["cu_seqlens"], src["pre-0001"]["cu_seqlens"])
    assert kw["scale"] == pytest.approx(src["pre-0001"]["scale"])
    kw2 = h.load_inputs(by["dec-0002"], root, device="cpu")
    assert kw2["state"] is None and kw2["q"].shape == (1, 1, 4, 128)


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.gpu
def test_run_records_on_gpu(gdn, dataset):
    root, src = dataset
    h = gdn.harness
    for rec in h.find_records(root):
        uuid = rec["workload"]["uuid"]
        out, ns = h.run_record(rec, root)
        torch.cuda.synchronize()
        s = src[uuid]
        st = s.get("state") if uuid != "dec-0002" else None
        args = (_bits(s["q"]), _bits(s["k"]), _bits(s["v"]), None if st is None else st.numpy(), s["A_log"].numpy(),
                _bits(s["a"]), s["dt_bias"].numpy(), _bits(s["b"]))
        if h.kind_of(rec["definition"]) == "decode":
            o_ref, s_ref = ref.decode(*args, s["scale"])
        else:
            o_ref, s_ref = ref.prefill(*args, s["cu_seqlens"].numpy(), s["scale"])
        np.testing.assert_allclose(out.float().cpu().numpy().reshape(-1), ref.bf16_bits_to_f32(o_ref).reshape(-1),
                                   atol=1e-2, rtol=1e-2)
        ok, err = state_close(ns.cpu().numpy(), s_ref, 1e-3)
        assert ok, (uuid, err)
        t = h.time_record(rec, root, warmup=1, iters=3)
        assert t["latency_ms"] > 0 and t["uuid"] == uuid
