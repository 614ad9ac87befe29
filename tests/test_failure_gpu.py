"""Device-side failure path on the GPU, without a fault: a bounded wait that runs out.

``GDN_FLAG_SELFTEST_WAIT_TIMEOUT`` makes every thread of a decode launch wait on a
barrier that nothing completes, with a 1 ms limit (no copy or tensor-core work is in
flight).  The waits give up, record ``GDN_DEVERR_WAIT_TIMEOUT`` and return; the host
reads the bit, and the same context then runs a normal decode that matches the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import state_close
from oracle import gdn_oracle as ref

pytestmark = pytest.mark.gpu


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def test_bounded_wait_gives_up_and_context_stays_usable(gdn):
    lib = gdn._lib
    inp = gdn.workloads.decode_inputs(4, seed=77)
    d = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}
    out = torch.full((4, 1, 32, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    ns = torch.full((4, 32, 128, 128), 7.0, dtype=torch.float32, device="cuda")
    lib.device_error(clear=True)
    gdn.kernel_decode.run_dps(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"],
                              d["scale"], out, ns, extra_flags=lib.GDN_FLAG_SELFTEST_WAIT_TIMEOUT)
    torch.cuda.synchronize()  # the launch ended by itself (every wait gave up after 1 ms)
    err = lib.device_error(clear=True)
    assert err & lib.GDN_DEVERR_WAIT_TIMEOUT, f"device error bits {err:#x}"
    assert bool((out == 7.0).all()) and bool((ns == 7.0).all()), "the aborted launch wrote outputs"
    # the context is intact: a normal decode on the same device matches the oracle
    out2, ns2 = gdn.kernel_decode.run(**d)
    torch.cuda.synchronize()
    o_ref, s_ref = ref.decode(bits(inp["q"]), bits(inp["k"]), bits(inp["v"]), inp["state"].numpy(),
                              inp["A_log"].numpy(), bits(inp["a"]), inp["dt_bias"].numpy(), bits(inp["b"]),
                              inp["scale"])
    np.testing.assert_allclose(out2.float().cpu().numpy(), ref.bf16_bits_to_f32(o_ref), atol=1e-2, rtol=1e-2)
    ok, e = state_close(ns2.cpu().numpy(), s_ref, 1e-3)
    assert ok, e
    assert lib.device_error(clear=True) == 0
