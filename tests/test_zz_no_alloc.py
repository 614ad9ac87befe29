"""``gdn_prefill_noalloc``: the prefill entry point that allocates nothing, for
callers that cannot allocate device memory at call time (code inside a captured or
pre-planned execution graph, or behind an allocator that must not grow).  Its
scratch (the prepared chunk records and the context-parallel segments' states and
maps) lives in a static device array inside the library.  Collected last, so it runs
both alone and after every other test."""
from __future__ import annotations

import pytest
import torch


def to_dev(inp):
    return {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}


def test_noalloc_rejects_problems_beyond_the_scratch(gdn):
    """Host-side size check, before anything is enqueued: 16 sequences of configs[3]
    size need ~357 MB of chunk records, and split into 15 segments each another
    16 x 32 x 40 states of 64 KB, far more than the 64 MiB scratch.  With the segment
    count forced by the flag the size does not depend on the device (the automatic
    count reads the SM count; without a GPU it assumes 148)."""
    lib = gdn._lib.library()
    N, T, HQ, HV, D = 16, 39332, 16, 32, 128
    flags = gdn._lib.GDN_PREFILL_SEGMENTS(15)
    need = lib.gdn_prefill_workspace_size(N, T, HQ, HV, D, flags)
    assert need > gdn._lib.GDN_PREFILL_NOALLOC_SCRATCH_BYTES
    rc = lib.gdn_prefill_noalloc(16, 4096, 128, 16, 4096, 128, 16, 8192, 128, None, 0, 0, 16, 16, 64, 16, 16, 64,
                                 16, 0, 0.0, 16, 8192, 128, 16, 32 * 16384, 16384, N, T, HQ, HV, D, flags, None)
    assert rc == gdn._lib.GDN_ERR_WORKSPACE
    assert "static scratch" in lib.gdn_last_error().decode()


@pytest.mark.gpu
@pytest.mark.parametrize("lens, segments", [([100, 64, 0, 257, 1, 700], 0), ([1500, 0, 700], 2)])
def test_noalloc_twice_matches_workspace_entry_point(gdn, lens, segments):
    """Two no-alloc calls in a row give the same outputs and states, bit for bit, as
    ``gdn_prefill`` with a caller workspace (same kernels, same inputs).  The second case
    forces 2 context-parallel segments, so the static scratch also holds segment states,
    maps and homogeneous outputs (after the records) that the calls must fully rewrite."""
    inp = to_dev(gdn.workloads.prefill_inputs(lens, seed=77))
    T, HV = inp["v"].shape[0], inp["v"].shape[1]
    N = inp["cu_seqlens"].shape[0] - 1
    args = [inp[k] for k in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens", "scale")]
    ref_out = torch.empty(T, HV, 128, dtype=torch.bfloat16, device="cuda")
    ref_state = torch.empty(N, HV, 128, 128, device="cuda")
    gdn.kernel_prefill.run_dps(*args, ref_out, ref_state, segments=segments)
    torch.cuda.synchronize()
    gdn._lib.device_error(clear=True)
    for _ in range(2):
        out = torch.full_like(ref_out, float("nan"))
        ns = torch.full_like(ref_state, float("nan"))
        gdn.kernel_prefill.run_dps(*args, out, ns, no_alloc=True, segments=segments)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out)
        assert torch.equal(ns, ref_state)
    assert gdn._lib.device_error() == 0
