"""The TVM-FFI route of the boundary (``libgdn_b200_tvm_ffi.so``).

CPU: the module loads, exports both operators, registers them as global functions,
and rejects host tensors before any CUDA call.  GPU: decode and prefill called
through the module (torch tensors via DLPack, torch's stream) match the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import state_close
from oracle import gdn_oracle as ref

tvm_ffi = pytest.importorskip("tvm_ffi")


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def test_module_exports_and_registers(gdn):
    mod = gdn.tvm_binding.module()
    assert mod.get_function("gdn_version")() == gdn._lib.library().gdn_version()
    names = gdn.tvm_binding.register(prefix="gdn_b200_test")
    assert set(names) == {"gdn_b200_test.decode", "gdn_b200_test.prefill"}
    for name in names:
        assert tvm_ffi.get_global_func(name) is not None


def test_host_tensors_are_rejected(gdn):
    inp = gdn.workloads.decode_inputs(2, seed=3)
    out = torch.empty(2, 1, 32, 128, dtype=torch.bfloat16)
    ns = torch.empty(2, 32, 128, 128)
    with pytest.raises(ValueError, match="must be on cuda"):
        gdn.tvm_binding.decode(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"],
                               inp["dt_bias"], inp["b"], None, out, ns)


@pytest.mark.gpu
def test_decode_through_tvm_ffi(gdn):
    inp = gdn.workloads.decode_inputs(5, seed=61)
    d = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}
    out = torch.empty(5, 1, 32, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(5, 32, 128, 128, device="cuda")
    with tvm_ffi.use_torch_stream():
        gdn.tvm_binding.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"],
                               None, out, ns)
    torch.cuda.synchronize()
    o_ref, s_ref = ref.decode(bits(inp["q"]), bits(inp["k"]), bits(inp["v"]), inp["state"].numpy(),
                              inp["A_log"].numpy(), bits(inp["a"]), inp["dt_bias"].numpy(), bits(inp["b"]), None)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.bf16_bits_to_f32(o_ref), atol=1e-2, rtol=1e-2)
    ok, err = state_close(ns.cpu().numpy(), s_ref, 1e-3)
    assert ok, err


@pytest.mark.gpu
def test_prefill_through_tvm_ffi_registered_global(gdn):
    gdn.tvm_binding.register()
    fn = tvm_ffi.get_global_func("gdn_b200.prefill")
    lens = [130, 0, 64, 7]
    inp = gdn.workloads.prefill_inputs(lens, seed=62)
    d = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}
    out = torch.empty(sum(lens), 32, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(len(lens), 32, 128, 128, device="cuda")
    with tvm_ffi.use_torch_stream():
        fn(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"], d["cu_seqlens"], None,
           out, ns)
    torch.cuda.synchronize()
    o_ref, s_ref = ref.prefill(bits(inp["q"]), bits(inp["k"]), bits(inp["v"]), inp["state"].numpy(),
                               inp["A_log"].numpy(), bits(inp["a"]), inp["dt_bias"].numpy(), bits(inp["b"]),
                               inp["cu_seqlens"].numpy(), None)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.bf16_bits_to_f32(o_ref), atol=1e-2, rtol=1e-2)
    ok, err = state_close(ns.cpu().numpy(), s_ref, 1e-3)
    assert ok, err
