"""Multi-GPU prefill shards on one GPU: every rank's share of a call, run through
``sharding.prefill_shard_calls`` (views of the full call's tensors: whole sequences,
or v-head pairs when there are fewer sequences than ranks), must rebuild the outputs
and final states of the single full call bit for bit.  Each (sequence, v-head)
chain is computed by the same kernels from the same inputs whichever rank owns it;
segments = 1 keeps the in-GPU segment count out of the comparison, and the automatic
segment count is checked against the oracle tolerances."""
from __future__ import annotations

import pytest
import torch

from conftest import state_close

pytestmark = pytest.mark.gpu


def run_shards(gdn, inp, lens, world, **kw):
    out = torch.full((sum(lens), 32, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
    ns = torch.full((len(lens), 32, 128, 128), float("nan"), device="cuda")
    for shard in gdn.sharding.plan_prefill(lens, 32, world):
        for c in gdn.sharding.prefill_shard_calls(shard, lens, inp["q"], inp["k"], inp["v"], inp["state"],
                                                  inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], out, ns):
            gdn.kernel_prefill.run_dps(**c, scale=inp["scale"], **kw)
    return out, ns


@pytest.mark.parametrize("lens,world", [([700, 130, 64, 1000, 5, 300], 4),   # whole sequences
                                        ([900, 257], 4),                        # v-head pairs (8 per rank)
                                        ([2000], 8)])                           # v-head pairs (4 per rank)
def test_shards_rebuild_the_full_prefill(gdn, lens, world):
    inp = gdn.workloads.prefill_inputs(lens, seed=71, device="cuda")
    full_o, full_s = gdn.kernel_prefill.run(**inp, segments=1)
    out, ns = run_shards(gdn, inp, lens, world, segments=1)
    assert torch.equal(out, full_o)
    assert torch.equal(ns, full_s)
    # with the library's own segment choice per shard: within the state tolerance of the full call
    out2, ns2 = run_shards(gdn, inp, lens, world)
    torch.testing.assert_close(out2.float(), full_o.float(), atol=1e-2, rtol=1e-2)
    ok, err = state_close(ns2.cpu().numpy(), full_s.cpu().numpy(), 1e-3)
    assert ok, err
    assert gdn._lib.device_error() == 0
