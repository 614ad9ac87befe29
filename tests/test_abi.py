"""The C-ABI library loads and exports every symbol ``include/gdn_b200.h``
declares; host-side validation rejects bad arguments before any launch.
CPU only: no call here reaches a kernel."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "gdn_b200.h"


@pytest.fixture(scope="module")
def lib(gdn):
    import importlib.util

    spec = importlib.util.spec_from_file_location("_gdn_build", Path(gdn.__file__).parent / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()
    return gdn._lib.library()


def declared_functions():
    text = HEADER.read_text()
    return re.findall(r"GDN_API\s+[\w\s\*]+?\b(gdn_\w+)\s*\(", text)


def test_header_declares_expected_entry_points():
    names = set(declared_functions())
    assert {"gdn_decode", "gdn_prefill", "gdn_prefill_workspace_size", "gdn_last_error",
            "gdn_device_error", "gdn_version"} <= names


def test_library_exports_every_declared_symbol(lib, gdn):
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in gdn._lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version(lib):
    assert lib.gdn_version() >= 100


def _decode_call(lib, **over):
    args = dict(q=8, k=8, v=8, state=None, A_log=16, a=8, dt_bias=16, b=8, out=8, new_state=16,
                B=1, HQ=16, HV=32, D=128, flags=0, qs=(2048, 128), ss=(32 * 16384, 16384))
    args.update(over)
    return lib.gdn_decode(args["q"], *args["qs"], args["k"], *args["qs"], args["v"], 4096, 128,
                          args["state"], *args["ss"], args["A_log"], args["a"], 32, args["dt_bias"],
                          args["b"], 32, 0.0, args["out"], 4096, 128, args["new_state"], *args["ss"],
                          args["B"], args["HQ"], args["HV"], args["D"], args["flags"], None)


@pytest.mark.parametrize("over,code,needle", [
    (dict(D=64), 2, "head_dim"),
    (dict(HV=24), 1, "multiple"),
    (dict(HQ=0), 1, "positive"),
    (dict(B=-1), 1, "batch"),
    (dict(flags=0x80), 1, "flag"),
    (dict(q=None), 1, "NULL"),
    (dict(new_state=None), 1, "new_state"),
    (dict(q=6), 2, "aligned"),
    (dict(new_state=8), 2, "16-byte"),
    (dict(state=16, new_state=16 + 64), 1, "overlap"),
])
def test_decode_rejects_bad_arguments(lib, over, code, needle):
    rc = _decode_call(lib, **over)
    assert rc == code
    assert needle in lib.gdn_last_error().decode()


def test_decode_batch_zero_is_a_no_op(lib):
    assert _decode_call(lib, B=0, q=None) == 0
    assert lib.gdn_last_error() == b""


def test_prefill_rejects_bad_arguments(lib):
    def call(**over):
        a = dict(cu=8, N=2, T=10, HQ=16, HV=32, D=128, ws=None, wsb=0, new_state=16)
        a.update(over)
        return lib.gdn_prefill(8, 2048, 128, 8, 2048, 128, 8, 4096, 128, None, 0, 0, 16, 8, 32, 16, 8, 32,
                               a["cu"], 0, 0.0, 8, 4096, 128, a["new_state"], 32 * 16384, 16384,
                               a["N"], a["T"], a["HQ"], a["HV"], a["D"], a["ws"], a["wsb"], 0, None)
    assert call(cu=None) == 1 and "cu_seqlens" in lib.gdn_last_error().decode()
    assert call(N=-1) == 1
    assert call(D=256) == 2
    assert call(N=0) == 0


def test_workspace_size(lib):
    """One 11,008-byte record (the lower triangle of T hi and lo + 7 gate arrays) per chunk slot and
    v-head; slots = total_tokens // 64 + num_seqs + 1.  In-kernel q/k normalisation
    adds one (1/|q|, log2 1/|q|) float pair per token and v-head after the records,
    256-byte aligned.  The forced token-serial path needs no workspace."""
    a = lib.gdn_prefill_workspace_size(16, 34000, 16, 32, 128, 0)
    assert a == lib.gdn_prefill_workspace_size(16, 34000, 16, 32, 128, 0)
    assert a == (34000 // 64 + 16 + 1) * 32 * 11008
    assert lib.gdn_prefill_workspace_size(8, 8 * 32768, 16, 32, 128, 0) == (4096 + 9) * 32 * 11008
    # GDN_FLAG_QK_L2NORM
    assert lib.gdn_prefill_workspace_size(16, 34000, 16, 32, 128, 0x1) == ((a + 255) & ~255) + 34000 * 32 * 8
    assert lib.gdn_prefill_workspace_size(16, 34000, 16, 32, 128, 0x2) == 0  # GDN_FLAG_PREFILL_SERIAL
    assert lib.gdn_prefill_workspace_size(0, 0, 16, 32, 128, 0) == 0


def test_workspace_size_with_segments(lib):
    """Context-parallel segments (S per sequence) add, after the records (256-byte aligned):
    [3][N][S - 1][HV] 64 KB states (the later segments' initial states, maps M and C), then
    Phi, the later segments' homogeneous outputs, [T][HV][128] bf16.  Automatic (no GPU here:
    148 SMs assumed): a plan is used when it beats one chain per (sequence, v-head) by 10 %;
    one 4096-token sequence with 32 v-heads (32 chains) gets 4 segments, two 8192-token
    sequences (64 chains) get 2 (segment 0 two thirds of the chunks, its chain beside the
    two map chains of the rest), many or short sequences none."""
    seg = lambda n: (n & 15) << 8  # noqa: E731  (GDN_PREFILL_SEGMENTS)
    rec = lambda n, t: (t // 64 + n + 1) * 32 * 11008  # noqa: E731
    phi = lambda t: t * 32 * 128 * 2  # noqa: E731
    st = 128 * 128 * 4
    assert lib.gdn_prefill_workspace_size(2, 3000, 16, 32, 128, seg(3)) == rec(2, 3000) + 3 * 2 * 2 * 32 * st + phi(3000)
    assert lib.gdn_prefill_workspace_size(2, 3000, 16, 32, 128, seg(2)) == rec(2, 3000) + 3 * 2 * 1 * 32 * st + phi(3000)
    assert lib.gdn_prefill_workspace_size(2, 3000, 16, 32, 128, seg(1)) == rec(2, 3000)
    assert lib.gdn_prefill_workspace_size(1, 4096, 16, 32, 128, 0) == rec(1, 4096) + 3 * 3 * 32 * st + phi(4096)
    assert lib.gdn_prefill_workspace_size(2, 8192, 16, 32, 128, 0) == rec(2, 8192) + 3 * 2 * 32 * st + phi(8192)
    assert lib.gdn_prefill_workspace_size(1, 512, 16, 32, 128, 0) == rec(1, 512)  # < 16 chunks
    assert lib.gdn_prefill_workspace_size(4, 4 * 8192, 16, 32, 128, 0) == rec(4, 4 * 8192)  # 128 chains
    # gdn_prefill_state_map (GDN_FLAG_STATE_MAP): records + [2][N][S][HV] segment maps; one long
    # 32-head sequence gets S = 2 (128 chains, one wave, half the chunks each)
    smap = 0x4
    assert lib.gdn_prefill_workspace_size(1, 4096, 16, 32, 128, smap) == rec(1, 4096) + 2 * 2 * 32 * st
    assert lib.gdn_prefill_workspace_size(1, 4096, 16, 32, 128, smap | seg(3)) == rec(1, 4096) + 2 * 3 * 32 * st
    assert lib.gdn_prefill_workspace_size(1, 4096, 16, 32, 128, smap | seg(1)) == rec(1, 4096)
    # 8 sequences: 512 map chains are 4 waves on 148 SMs, 1024 half-length ones 7 (= 3.5)
    assert lib.gdn_prefill_workspace_size(8, 8 * 4096, 16, 32, 128, smap) == rec(8, 8 * 4096) + 2 * 2 * 8 * 32 * st
    assert lib.gdn_prefill_workspace_size(8, 8 * 512, 16, 32, 128, smap) == rec(8, 8 * 512)  # 8 chunks each


def test_missing_library_fails_loudly(gdn, monkeypatch, tmp_path):
    monkeypatch.setattr(gdn._lib, "_lib", None)
    monkeypatch.setenv("GDN_B200_LIB", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="not built"):
        gdn._lib.library()


def test_cpu_tensors_are_rejected(gdn):
    import torch

    inp = gdn.workloads.decode_inputs(1)
    with pytest.raises(RuntimeError, match="CUDA"):
        gdn.kernel_decode.run(**inp)


def test_decode_pooled_rejects_bad_arguments(lib):
    def call(**over):
        a = dict(pool=16, idx=8, B=2, T=3, P=4, HQ=16, HV=32, D=128, new_pool=16, out=8, flags=0)
        a.update(over)
        return lib.gdn_decode_pooled(8, 3 * 2048, 2048, 128, 8, 3 * 2048, 2048, 128, 8, 3 * 4096, 4096, 128,
                                     a["pool"], 32 * 16384, 16384, a["idx"], 0,
                                     16, 8, 96, 32, 16, 8, 96, 32, 0.0,
                                     a["out"], 3 * 4096, 4096, 128, a["new_pool"], 32 * 16384, 16384,
                                     None, 0, 0, 0, a["B"], a["T"], a["P"], a["HQ"], a["HV"], a["D"], a["flags"], None)
    assert call(P=0) == 1 and "pool_size" in lib.gdn_last_error().decode()
    assert call(idx=None) == 1
    assert call(new_pool=None) == 1
    assert call(new_pool=24) == 2  # not 16-byte aligned
    assert call(pool=16, new_pool=16 + 1024) == 1 and "overlap" in lib.gdn_last_error().decode()
    assert call(D=64) == 2
    assert call(flags=0x2) == 1
    assert call(B=0) == 0 and call(T=0) == 0


def test_range_workspace_size(lib):
    """gdn_prefill_range_affine / _finish (GDN_FLAG_RANGE_AFFINE): records, then [3][N][S - 1][HV]
    64 KB states (every segment of the range is a map pair: S - 1 of them), then the homogeneous
    outputs [T][HV][128] bf16.  Automatic pair count (148 SMs assumed without a GPU): one
    16,384-token range of 32 v-heads gets 2 (128 CTAs of half a range in one wave); forced with
    GDN_PREFILL_SEGMENTS(n)."""
    ra, seg = 0x8, (lambda n: (n & 15) << 8)  # noqa: E731
    st = 128 * 128 * 4
    rec = (16384 // 64 + 1 + 1) * 32 * 11008
    phi = 16384 * 32 * 256
    assert lib.gdn_prefill_workspace_size(1, 16384, 16, 32, 128, ra) == rec + 3 * 2 * 32 * st + phi
    assert lib.gdn_prefill_workspace_size(1, 16384, 16, 32, 128, ra | seg(1)) == rec + 3 * 1 * 32 * st + phi
    assert lib.gdn_prefill_workspace_size(1, 16384, 16, 32, 128, ra | seg(4)) == rec + 3 * 4 * 32 * st + phi


def test_range_calls_reject_bad_arguments(lib):
    def affine(**over):
        a = dict(ws=None, wsb=0, flags=0x8, mm=16, out=16)
        a.update(over)
        return lib.gdn_prefill_range_affine(16, 2048, 128, 16, 2048, 128, 16, 4096, 128, 16, 8, 32, 16, 8, 32,
                                            8, 0, 0.0, a["out"], 4096, 128, a["mm"], 32 * 16384, 16384,
                                            16, 32 * 16384, 16384, 1, 640, 16, 32, 128, a["ws"], a["wsb"],
                                            a["flags"], None)
    assert affine(flags=0x8 | 0x1) == 1 and "flag" in lib.gdn_last_error().decode()  # no q/k L2 norm here
    assert affine(mm=None) == 1
    assert affine(out=24) == 2  # not 16-byte aligned
    assert affine() == 4 and "workspace" in lib.gdn_last_error().decode()

    def finish(**over):
        a = dict(state=None, prev=None, nprev=0, ns=16, ws=None, wsb=0)
        a.update(over)
        return lib.gdn_prefill_range_finish(8, 0, a["state"], 32 * 16384, 16384, a["prev"], a["nprev"],
                                            16, 4096, 128, a["ns"], 32 * 16384, 16384, 1, 640, 16, 32, 128,
                                            a["ws"], a["wsb"], 0x8, None)
    assert finish(state=16, prev=16, nprev=2) == 1 and "not both" in lib.gdn_last_error().decode()
    assert finish(nprev=-1) == 1
    assert finish(prev=None, nprev=1) == 1
    assert finish(ns=None) == 1
    assert finish() == 4
