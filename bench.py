"""Benchmark of the GDN hot path (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode_b64|decode_b1024|prefill_varlen16|prefill_8x32768|mtp_b64_t4]

Headline (``value``): GDN decode state GB/s on configs[1] (B = 64 sequences,
16 q/k heads, 32 v heads, d = 128, fp32 k-last state) per GPU; with N GPUs
each rank owns its own 64 sequences and states (weak scaling, no collective),
``value`` = algorithmic bytes of all ranks / max-over-ranks time.  A step is
one decode call over the batch; inputs are resident in HBM and rotate over
several buffer sets whose footprint exceeds 3x L2 (126 MB), so no step reads
L2-resident state.  ``e2e`` times the public ``run()`` with host (pinned)
inputs and outputs, copies included.

Further legs of the same line (each with its own CUDA-event timing, roofline and
clock record): ``decode_b1024`` = configs[2] (1024 sequences split over the N
ranks, strong scaling), ``prefill`` = configs[3] (varlen, 16 sequences, on every
rank), ``prefill_8x32768`` = configs[4] (8 x 32768 tokens split over the ranks by
sequence, strong scaling), ``mtp`` = pooled multi-token decode (64 sequences x 4
tokens, in-place state pool; ``--workload mtp_b64_t4`` adds the same call at 1 .. 8
tokens per sequence as ``tokens_sweep``).  At N = 1 rank 0 also times the CPU baselines (the
C restatement of the reference recurrence for decode and prefill, and the
flashinfer torch reference recurrence) and ``reference_triton``: the reference's
own Triton kernels (``solution/triton/kernel_{decode,prefill}.py::run``,
unmodified, staged in ``baseline/_ref``) on this GPU beside this library, on
configs[1], configs[3] and the reference's own qk4/v8 shapes.

``--impl reference`` times the reference algorithm's CPU implementation (the
C restatement in ``oracle/``, all host threads) on a bounded sample of the
same workload and prints the same line with ``"impl": "reference"``.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from __graft_entry__ import load_package  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


# ----------------------------------------------------------------------------- helpers
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", 0)), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, FALLBACK_BF16_TFLOPS, "fallback"


def profile_traffic(name: str):
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of the
    kernel as recorded from an ncu capture in ``profiles/<name>.txt``."""
    p = ROOT / "profiles" / f"{name}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1].split()[0])
    return None


class ClockSampler:
    """Samples SM clocks and clock-event reasons with NVML during the timed region."""
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples, self.reasons, self.period = [], 0, period_s
        self._stop = threading.Event()
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report no clocks
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._nv is not None:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml_unavailable"]}
        reasons = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world} (launch N>1 with torchrun)")
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ----------------------------------------------------------------------------- workloads
def decode_sets(gdn, batch, n_sets, seed, device):
    sets = []
    for i in range(n_sets):
        inp = gdn.workloads.decode_inputs(batch, seed=seed + 1000 * i, device=device)
        inp["output"] = torch.empty(batch, 1, 32, 128, dtype=torch.bfloat16, device=device)
        inp["new_state"] = torch.empty_like(inp["state"])
        sets.append(inp)
    return sets


def decode_call(gdn, s):
    gdn.kernel_decode.run_dps(s["q"], s["k"], s["v"], s["state"], s["A_log"], s["a"], s["dt_bias"],
                              s["b"], s["scale"], s["output"], s["new_state"])


def prefill_sets(gdn, seqlens, n_sets, seed, device, zero_state=False):
    sets = []
    for i in range(n_sets):
        inp = gdn.workloads.prefill_inputs(seqlens, seed=seed + 1000 * i, device=device,
                                           zero_state=zero_state)
        T = sum(seqlens)
        inp["output"] = torch.empty(T, 32, 128, dtype=torch.bfloat16, device=device)
        inp["new_state"] = torch.empty_like(inp["state"])
        if zero_state:
            inp["state"] = None
        sets.append(inp)
    return sets


def prefill_launches(gdn, seqlens):
    """Kernels one prefill step launches: prep + chain, or with the automatic in-GPU
    segments prep + pass 1 (segment 0 and the later segments' maps) + the map
    composition + the output correction; segments show as extra workspace."""
    N, T = len(seqlens), sum(seqlens)
    auto = gdn.kernel_prefill.workspace_size(N, T, 16, 32)
    one = gdn.kernel_prefill.workspace_size(N, T, 16, 32, segments=1)
    return 2 if auto <= one else 4


def prefill_call(gdn, s, use_qk_l2norm=False):
    gdn.kernel_prefill.run_dps(s["q"], s["k"], s["v"], s["state"], s["A_log"], s["a"], s["dt_bias"],
                               s["b"], s["cu_seqlens"], s["scale"], s["output"], s["new_state"],
                               use_qk_l2norm=use_qk_l2norm)


def mtp_sets(gdn, batch, tokens, n_sets, seed, device):
    """Pooled multi-token decode: one state pool of batch * n_sets slots (in-place
    serving update), n_sets disjoint index sets so consecutive steps touch
    different slots (pool > 3x L2)."""
    P = batch * n_sets
    gen = torch.Generator().manual_seed(seed)
    pool = (torch.randn(P, 32, 128, 128, generator=gen) * 0.05).to(device)
    perm = torch.randperm(P, generator=gen)
    sets = []
    for i in range(n_sets):
        inp = gdn.workloads.prefill_inputs([tokens] * batch, seed=seed + 1000 * i, device=device)
        rs = lambda t: t.reshape(batch, tokens, *t.shape[1:])  # noqa: E731
        sets.append(dict(q=rs(inp["q"]), k=rs(inp["k"]), v=rs(inp["v"]), a=rs(inp["a"]), b=rs(inp["b"]),
                         A_log=inp["A_log"], dt_bias=inp["dt_bias"], pool=pool,
                         idx=perm[i * batch:(i + 1) * batch].to(device=device, dtype=torch.int32),
                         output=torch.empty(batch, tokens, 32, 128, dtype=torch.bfloat16, device=device)))
    return sets


def mtp_call(gdn, s):
    gdn.kernel_mtp.run_dps(s["q"], s["k"], s["v"], s["pool"], s["idx"], s["A_log"], s["a"], s["dt_bias"], s["b"],
                           None, s["output"], s["pool"])


def set_bytes(s):
    return sum(v.numel() * v.element_size() for v in s.values() if torch.is_tensor(v))


def time_steps(call, sets, steps, warmup, world, sampler=None, graph=False):
    """Warm up, then time exactly ``steps`` calls bracketed by barrier +
    synchronize, with CUDA events on the launching stream around the timed region
    only (events recorded between the steps would add their own gaps to it).
    With ``graph`` the ``steps`` calls are captured once into a CUDA graph (the
    serving form of a decode loop) and the timed region is one replay of it; the
    first replay, untimed, uploads the graph.  Returns (ms per step, max over
    ranks; this rank's ms per step = the average duration of one step's launches)."""
    stream = torch.cuda.current_stream()
    for i in range(warmup):
        call(sets[i % len(sets)])
    g = None
    if graph:
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(steps):
                call(sets[i % len(sets)])
        g.replay()
        torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    ctx = sampler if sampler is not None else _Null()
    with ctx:
        t0.record(stream)
        if g is not None:
            g.replay()
        else:
            for i in range(steps):
                call(sets[i % len(sets)])
        t1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    total_ms = t0.elapsed_time(t1)
    del g
    return max_over_ranks(total_ms, world) / steps, total_ms / steps


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


# ----------------------------------------------------------------------------- e2e
def decode_e2e(gdn, batch, steps, warmup, world, seed):
    """Public API with host buffers: every step copies its inputs (the state
    included) from pinned host memory to the device, runs the decode
    (``kernel_decode.run_dps``) and copies the output and the new state back to
    pinned host memory.  Copies in, compute and copies out run on three streams
    over two device buffer sets, so step i's inputs go up while step i - 1's
    results come down (the two PCIe directions overlap, as in a serving loop)."""
    host = gdn.workloads.decode_inputs(batch, seed=seed)
    names = [k for k, v in host.items() if torch.is_tensor(v)]
    pinned = {k: host[k].pin_memory() for k in names}
    scale = host["scale"]
    out_h = torch.empty(batch, 1, 32, 128, dtype=torch.bfloat16).pin_memory()
    st_h = torch.empty(batch, 32, 128, 128, dtype=torch.float32).pin_memory()
    dev = [{k: torch.empty_like(pinned[k], device="cuda") for k in names} for _ in range(2)]
    outs = [(torch.empty(batch, 1, 32, 128, dtype=torch.bfloat16, device="cuda"),
             torch.empty(batch, 32, 128, 128, dtype=torch.float32, device="cuda")) for _ in range(2)]
    s_comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]    # inputs of buffer set b are on the device
    ev_comp = [torch.cuda.Event() for _ in range(2)]  # the decode on set b is done (inputs read)
    ev_out = [torch.cuda.Event() for _ in range(2)]   # the results of set b are back on the host
    used = [False, False]
    h2d = sum(pinned[k].numel() * pinned[k].element_size() for k in names)
    d2h = out_h.numel() * 2 + st_h.numel() * 4

    def step(i):
        b = i % 2
        d = dev[b]
        if used[b]:
            s_in.wait_event(ev_comp[b])
        with torch.cuda.stream(s_in):
            for k in names:
                d[k].copy_(pinned[k], non_blocking=True)
        ev_in[b].record(s_in)
        s_comp.wait_event(ev_in[b])
        if used[b]:
            s_comp.wait_event(ev_out[b])
        gdn.kernel_decode.run_dps(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"],
                                  scale, outs[b][0], outs[b][1])
        ev_comp[b].record(s_comp)
        s_out.wait_event(ev_comp[b])
        with torch.cuda.stream(s_out):
            out_h.copy_(outs[b][0], non_blocking=True)
            st_h.copy_(outs[b][1], non_blocking=True)
        ev_out[b].record(s_out)
        used[b] = True

    for i in range(warmup):
        step(i)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    t0.record(s_in)
    for i in range(steps):
        step(warmup + i)
    t1.record(s_out)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(t0.elapsed_time(t1), world) / steps, h2d, d2h


# ----------------------------------------------------------------------------- CPU legs
def cpu_decode_rate(gdn, batch, budget_s, nthreads=None):
    """C restatement of the reference recurrence on the host cores; returns
    (GB/s, sample description, cores)."""
    import numpy as np

    from oracle import c_oracle

    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    inp = gdn.workloads.decode_inputs(batch, seed=0)
    args = (bits(inp["q"]), bits(inp["k"]), bits(inp["v"]), inp["state"].numpy(), inp["A_log"].numpy(),
            bits(inp["a"]), inp["dt_bias"].numpy(), bits(inp["b"]), inp["scale"])
    cores = nthreads or c_oracle.default_threads()
    c_oracle.decode(*args, nthreads=cores)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        c_oracle.decode(*args, nthreads=cores)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    gb = gdn.workloads.decode_bytes_per_seq() * batch * reps / 1e9
    return gb / el, f"{reps} full decode steps of B={batch} (16/32 heads) in {el:.1f} s", cores


def cpu_prefill_rate(gdn, seqlens, budget_s, nthreads=None):
    """Tokens/s of the C restatement on a sample: the first tokens of every sequence
    (time-bounded by doubling the per-sequence prefix until the budget is used)."""
    import numpy as np

    from oracle import c_oracle

    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    cores = nthreads or c_oracle.default_threads()
    prefix, best = 16, None
    while True:
        lens = [min(prefix, L) for L in seqlens]
        inp = gdn.workloads.prefill_inputs(lens, seed=0)
        args = (bits(inp["q"]), bits(inp["k"]), bits(inp["v"]), inp["state"].numpy(),
                inp["A_log"].numpy(), bits(inp["a"]), inp["dt_bias"].numpy(), bits(inp["b"]),
                inp["cu_seqlens"].numpy(), inp["scale"])
        t0 = time.perf_counter()
        c_oracle.prefill(*args, nthreads=cores)
        el = time.perf_counter() - t0
        best = (sum(lens) / el, f"first {prefix} tokens of each of {len(lens)} sequences "
                                f"({sum(lens)} tokens) in {el:.1f} s", cores)
        if el * 2.5 > budget_s or prefix >= max(seqlens):
            return best
        prefix *= 2


def cpu_mtp_rate(gdn, batch, tokens, budget_s, nthreads=None):
    """State GB/s of the C restatement on the pooled multi-token decode: each
    sequence is ``tokens`` steps of the recurrence from its slot (run as a varlen
    prefill of ``batch`` sequences of ``tokens`` tokens, which is the same
    arithmetic); returns (GB/s, sample description, cores)."""
    import numpy as np

    from oracle import c_oracle

    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    cores = nthreads or c_oracle.default_threads()
    inp = gdn.workloads.prefill_inputs([tokens] * batch, seed=0)
    args = (bits(inp["q"]), bits(inp["k"]), bits(inp["v"]), inp["state"].numpy(), inp["A_log"].numpy(),
            bits(inp["a"]), inp["dt_bias"].numpy(), bits(inp["b"]), inp["cu_seqlens"].numpy(), inp["scale"])
    c_oracle.prefill(*args, nthreads=cores)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        c_oracle.prefill(*args, nthreads=cores)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    gb = gdn.workloads.mtp_bytes_per_seq(tokens) * batch * reps / 1e9
    return gb / el, f"{reps} calls of B={batch} x T={tokens} tokens (16/32 heads) in {el:.1f} s", cores


# ----------------------------------------------------------------------------- legs
def leg_steps(steps: int, cap: int, floor: int = 10) -> int:
    """Timed steps of a secondary leg: the run's K, capped so the default run stays short."""
    return max(floor, min(steps, cap))


def decode_leg(gdn, wl, world, rank, local, steps, warmup, peaks, with_e2e):
    """configs[1] (``decode_b64``: 64 sequences per rank, weak scaling) or configs[2]
    (``decode_b1024``: 1024 sequences split over the ranks, strong scaling)."""
    hbm_peak, _, _, peak_kind = peaks
    if wl == "decode_b64":
        batch = 64
    else:
        lo, hi = gdn.sharding.batch_slice(1024, world, rank)
        batch = hi - lo
    one = decode_sets(gdn, batch, 1, seed=rank, device="cuda")
    n_sets = max(2, math.ceil(3 * L2_BYTES / set_bytes(one[0])))
    sets = one + decode_sets(gdn, batch, n_sets - 1, seed=rank + 1, device="cuda")
    sampler = ClockSampler(local)
    ms, launch_ms = time_steps(lambda s: decode_call(gdn, s), sets, steps, warmup, world, sampler, graph=True)
    bytes_rank = gdn.workloads.decode_bytes_per_seq() * batch
    total_bytes = sum_over_ranks(bytes_rank, world)
    achieved = bytes_rank / (launch_ms * 1e-3) / 1e9
    res = dict(
        workload=wl, gbs=total_bytes / (ms * 1e-3) / 1e9,
        tokens_per_s=sum_over_ranks(batch, world) / (ms * 1e-3), ms_per_step=ms, steps=steps,
        batch_per_rank=batch, rotating_buffer_sets=len(sets),
        l2=f"inputs larger than L2: {len(sets)} rotating sets, {len(sets) * set_bytes(sets[0]) / 1e6:.0f} MB footprint",
        scaling="weak" if wl == "decode_b64" else "strong",
        roofline={"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                  "frac": achieved / hbm_peak, "peak_kind": f"{peak_kind} hbm_gbs (copy, burst)",
                  "traffic": profile_traffic(f"gdn_{wl}"), "kernel": "decode_kernel",
                  "avg_launch_us": launch_ms * 1e3, "algorithmic_bytes_per_launch": bytes_rank},
        clocks=sampler.summary())
    del sets
    if with_e2e:
        e2e_steps = leg_steps(steps, 50, floor=20)
        e2e_ms, h2d, d2h = decode_e2e(gdn, batch, e2e_steps, 3, world, seed=rank)
        res["e2e"] = {"value": total_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                      "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "steps": e2e_steps,
                      "path": "kernel_decode.run_dps() with pinned host inputs and outputs (state in and out "
                              "every step); copies in, decode and copies out on three streams over two device "
                              "buffer sets"}
    torch.cuda.empty_cache()
    return res


def prefill_leg(gdn, wl_p, world, rank, local, steps, warmup, peaks):
    """configs[3] (``prefill_varlen16``, the whole batch on every rank) or configs[4]
    (``prefill_8x32768``, sequences split over the ranks: strong scaling)."""
    _, bf16_peak, _, peak_kind = peaks
    cfg = gdn.workloads.config(3 if wl_p == "prefill_varlen16" else 4)
    seqlens = list(cfg.seqlens)
    if wl_p == "prefill_8x32768" and world > 1:
        plan = gdn.sharding.plan_prefill(seqlens, 32, world)
        seqlens = [seqlens[i] for i in plan[rank].seqs]
    psets = prefill_sets(gdn, seqlens, 2, seed=rank, device="cuda", zero_state=cfg.zero_state)
    sampler = ClockSampler(local)
    pms, plaunch = time_steps(lambda s: prefill_call(gdn, s), psets, steps, warmup, world, sampler)
    tokens = sum_over_ranks(sum(seqlens), world)
    flops_launch = gdn.workloads.prefill_flops_per_token() * sum(seqlens)
    traffic = profile_traffic(f"gdn_{wl_p}")
    res = {"workload": wl_p, "tokens_per_s": tokens / (pms * 1e-3), "ms_per_step": pms, "steps": steps,
           "tokens_per_rank": sum(seqlens), "num_seqs_per_rank": len(seqlens),
           "scaling": "strong" if wl_p == "prefill_8x32768" else "weak",
           "roofline": {"bound": "tensor", "achieved": flops_launch / (plaunch * 1e-3) / 1e12,
                        "peak": bf16_peak, "unit": "TFLOP/s",
                        "frac": flops_launch / (plaunch * 1e-3) / 1e12 / bf16_peak,
                        "peak_kind": f"{peak_kind} bf16_tflops (burst)",
                        "kernel": "one prefill step (every kernel of the call): algorithmic FLOPs / step time",
                        "hbm_gbs": gdn.workloads.prefill_bytes(sum(seqlens), len(seqlens)) / (plaunch * 1e-3) / 1e9,
                        "traffic": traffic,
                        "traffic_source": f"profiles/gdn_{wl_p}.txt" if traffic is not None else None,
                        "avg_launch_us": plaunch * 1e3},
           "gpu_launches_per_step": prefill_launches(gdn, seqlens),
           "clocks": sampler.summary()}
    if wl_p == "prefill_varlen16":
        # the same step with q and k L2-normalised inside the kernels (use_qk_l2norm)
        lms, _ = time_steps(lambda s: prefill_call(gdn, s, use_qk_l2norm=True), psets, steps, warmup, world)
        res["qk_l2norm"] = {"tokens_per_s": tokens / (lms * 1e-3), "ms_per_step": lms,
                            "relative_to_default": pms / lms}
    del psets
    torch.cuda.empty_cache()
    return res, seqlens


def cpu_torch_reference(budget_s: float):
    """The definition's torch reference recurrence (flashinfer 0.6.11.post2,
    ``flashinfer/trace/templates/gdn.py``) on the host cores: configs[0] (decode B = 1)
    and a prefill sample.  Returns a dict, or the reason it could not run."""
    try:
        from flashinfer.trace.templates.gdn import _gdn_decode_reference, _gdn_prefill_reference
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"flashinfer torch reference not importable: {type(e).__name__}: {e}"[:200]}
    gdn = load_package()
    cores = os.cpu_count() or 1
    old = torch.get_num_threads()
    torch.set_num_threads(cores)
    try:
        inp = gdn.workloads.decode_inputs(1, seed=0)
        args = (inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"],
                inp["scale"])
        _gdn_decode_reference(*args)
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s / 2:
            _gdn_decode_reference(*args)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        dec = {"workload": "configs[0] decode B=1", "ms_per_step": dt * 1e3,
               "gbs": gdn.workloads.decode_bytes_per_seq() / dt / 1e9, "reps": reps}
        pin = gdn.workloads.prefill_inputs([64], seed=0)
        pargs = (pin["q"], pin["k"], pin["v"], pin["state"], pin["A_log"], pin["a"], pin["dt_bias"], pin["b"],
                 pin["cu_seqlens"], pin["scale"])
        t0 = time.perf_counter()
        _gdn_prefill_reference(*pargs)
        dt = time.perf_counter() - t0
        pre = {"workload": "prefill sample: 1 sequence x 64 tokens (16/32 heads)", "tokens_per_s": 64 / dt,
               "seconds": dt}
        return {"impl": "flashinfer 0.6.11.post2 _gdn_decode_reference / _gdn_prefill_reference (torch, CPU)",
                "cores": cores, "torch_threads": cores, "decode": dec, "prefill": pre}
    finally:
        torch.set_num_threads(old)


def _load_by_path(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _time_graph(call, sets, steps, warmup):
    """Device time per call: ``steps`` calls captured into one CUDA graph (first replay
    untimed), CUDA events around one replay; eager back-to-back calls if capture fails."""
    stream = torch.cuda.current_stream()
    for i in range(warmup):
        call(sets[i % len(sets)])
    torch.cuda.synchronize()
    g, how = None, "graph"
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(steps):
                call(sets[i % len(sets)])
        g.replay()
        torch.cuda.synchronize()
    except Exception:  # noqa: BLE001
        g, how = None, "eager"
        torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record(stream)
    if g is not None:
        g.replay()
    else:
        for i in range(steps):
            call(sets[i % len(sets)])
    t1.record(stream)
    torch.cuda.synchronize()
    del g
    return t0.elapsed_time(t1) / steps, how


def qk4v8_prefill_lens(total: int = 8192, num_seqs: int = 32, seed: int = 8):
    """A seeded multi-sequence prefill of ``total`` tokens, like the reference's
    8192-token workloads (20-57 sequences)."""
    gen = torch.Generator().manual_seed(seed)
    w = torch.rand(num_seqs, generator=gen) + 0.05
    lens = [max(1, int(x)) for x in (w / w.sum() * total)]
    lens[-1] += total - sum(lens)
    return lens


def reference_triton_leg(gdn, steps):
    """The reference's own sm_100 Triton kernels on this GPU beside this library, same
    inputs and the same timing protocol (value-returning ``run`` of both, K calls in one
    CUDA graph, rotating input sets larger than L2 where the state is large)."""
    root = ROOT / "baseline" / "_ref" / "solution" / "triton"
    if not (root / "kernel_decode.py").exists():
        return {"unavailable": "reference Triton kernels not staged in baseline/_ref (run __graft_entry__.build() "
                               "where the reference checkout is present)"}
    try:
        import triton  # noqa: F401
        kd = _load_by_path("gdn_ref_kernel_decode", root / "kernel_decode.py")
        kp = _load_by_path("gdn_ref_kernel_prefill", root / "kernel_prefill.py")
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference Triton kernels do not load on this box: {type(e).__name__}: {e}"[:300]}
    K = max(10, min(steps, 50))
    out = {"source": "solution/triton/kernel_decode.py::run, kernel_prefill.py::run (unmodified, staged copy)",
           "timing": f"{K} calls of each arm's value-returning run() captured in one CUDA graph, CUDA events "
                     "around one replay (eager back-to-back calls if capture fails)"}

    def dec_case(name, B, HQ, HV):
        one = gdn.workloads.decode_inputs(B, num_qk_heads=HQ, num_v_heads=HV, seed=3, device="cuda")
        per_set = sum(v.numel() * v.element_size() for v in one.values() if torch.is_tensor(v))
        n = max(2, math.ceil(3 * L2_BYTES / per_set))
        sets = [one] + [gdn.workloads.decode_inputs(B, num_qk_heads=HQ, num_v_heads=HV, seed=3 + i, device="cuda")
                        for i in range(1, n)]
        keys = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "scale")
        ref_ms, ref_how = _time_graph(lambda s: kd.run(*[s[k] for k in keys]), sets, K, 3)
        our_ms, our_how = _time_graph(lambda s: gdn.kernel_decode.run(*[s[k] for k in keys]), sets, K, 3)
        nbytes = gdn.workloads.decode_bytes_per_seq(HQ, HV) * B
        out[name] = {"batch": B, "heads_qk_v": [HQ, HV], "rotating_sets": n,
                     "reference_us": ref_ms * 1e3, "ours_us": our_ms * 1e3,
                     "reference_gbs": nbytes / (ref_ms * 1e-3) / 1e9, "ours_gbs": nbytes / (our_ms * 1e-3) / 1e9,
                     "speedup": ref_ms / our_ms, "capture": [ref_how, our_how]}
        del sets
        torch.cuda.empty_cache()

    def pre_case(name, lens, HQ, HV):
        sets = [gdn.workloads.prefill_inputs(lens, num_qk_heads=HQ, num_v_heads=HV, seed=5 + i, device="cuda")
                for i in range(2)]
        keys = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens", "scale")
        kk = max(3, K // 5)
        ref_ms, ref_how = _time_graph(lambda s: kp.run(*[s[k] for k in keys]), sets, kk, 2)
        our_ms, our_how = _time_graph(lambda s: gdn.kernel_prefill.run(*[s[k] for k in keys]), sets, kk, 2)
        T = sum(lens)
        out[name] = {"num_seqs": len(lens), "tokens": T, "heads_qk_v": [HQ, HV],
                     "reference_ms": ref_ms, "ours_ms": our_ms,
                     "reference_tokens_per_s": T / (ref_ms * 1e-3), "ours_tokens_per_s": T / (our_ms * 1e-3),
                     "speedup": ref_ms / our_ms, "capture": [ref_how, our_how]}
        del sets
        torch.cuda.empty_cache()

    try:
        dec_case("configs1_decode_b64", 64, 16, 32)
        for B in (1, 8, 64):
            dec_case(f"qk4v8_decode_b{B}", B, 4, 8)
        pre_case("configs3_prefill_varlen16", list(gdn.workloads.config(3).seqlens), 16, 32)
        pre_case("qk4v8_prefill_8192", qk4v8_prefill_lens(), 4, 8)
    except Exception as e:  # noqa: BLE001
        out["error"] = f"{type(e).__name__}: {e}"[:300]
    return out


# ----------------------------------------------------------------------------- main
def run_reference(args, world, rank):
    """Reference arm: the reference algorithm's CPU implementation (the C
    restatement, all host threads), same metric.  Each step is a bounded sample
    of the workload: ``m`` of its sequences, with ``m`` sized so the whole
    ``--steps/--warmup`` run takes about a minute."""
    if rank != 0:
        return
    import numpy as np

    from oracle import c_oracle

    gdn = load_package()
    batch = 64 if args.workload == "decode_b64" else 1024
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    inp = gdn.workloads.decode_inputs(batch, seed=0)
    cores = c_oracle.default_threads()

    def args_for(m):
        return (bits(inp["q"][:m]), bits(inp["k"][:m]), bits(inp["v"][:m]), inp["state"][:m].numpy(),
                inp["A_log"].numpy(), bits(inp["a"][:m]), inp["dt_bias"].numpy(), bits(inp["b"][:m]),
                inp["scale"])

    probe = args_for(min(batch, cores))
    c_oracle.decode(*probe, nthreads=cores)
    t0 = time.perf_counter()
    c_oracle.decode(*probe, nthreads=cores)
    per_seq = (time.perf_counter() - t0) / min(batch, cores)
    per_step_budget = 60.0 / max(1, args.steps + args.warmup)
    m = max(1, min(batch, int(per_step_budget / max(per_seq, 1e-9))))
    sample = args_for(m)
    vals = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        c_oracle.decode(*sample, nthreads=cores)
        el = time.perf_counter() - t0
        if i >= args.warmup:
            vals.append(gdn.workloads.decode_bytes_per_seq() * m / el / 1e9)
    value = statistics.median(vals)
    bytes_step = gdn.workloads.decode_bytes_per_seq() * batch
    line = {
        "impl": "reference", "metric": "GDN decode state GB/s", "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": bytes_step / (value * 1e9) * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE distributions)",
        "config": {"workload": args.workload, "batch_per_rank": batch, "num_qk_heads": 16,
                   "num_v_heads": 32, "head_dim": 128, "state": "fp32 k-last"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"each step: {m} of the {batch} sequences (all 32 heads); median over "
                                   f"{args.steps} steps; C restatement of the reference recurrence"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    gdn = load_package()
    peaks = measured_peaks()
    hbm_peak, bf16_peak, bf16_sust, peak_kind = peaks
    wl = args.workload
    result = {}
    legs = args.legs and wl == "decode_b64"
    leg_warm = max(3, min(args.warmup, 10))
    if wl.startswith("decode"):
        d = decode_leg(gdn, wl, world, rank, local, args.steps, args.warmup, peaks, with_e2e=True)
        cfg = {"workload": wl, "batch_per_rank": d["batch_per_rank"], "num_qk_heads": 16, "num_v_heads": 32,
               "head_dim": 128, "state": "fp32 k-last", "rotating_buffer_sets": d["rotating_buffer_sets"],
               "l2": d["l2"], "parallelism": f"dp{world} (sequences sharded, no collective)",
               "timing": "the K steps replayed from one CUDA graph (the serving form of a decode loop); "
                         "CUDA events around the timed region only"}
        result.update(metric="GDN decode state GB/s", value=d["gbs"], unit="GB/s", ms_per_step=d["ms_per_step"],
                      dtype="f32", config=cfg, roofline=d["roofline"], e2e=d["e2e"], gpu_launches=args.steps,
                      clocks=d["clocks"], scaling=d["scaling"])
        if legs:
            result["decode_b1024"] = decode_leg(gdn, "decode_b1024", world, rank, local, leg_steps(args.steps, 200),
                                                leg_warm, peaks, with_e2e=False)
    if legs or wl == "mtp_b64_t4":
        # pooled multi-token decode (serving form): 64 sequences x 4 tokens per call, in place
        mb, mt = 64, 4
        msets = mtp_sets(gdn, mb, mt, 3, seed=rank + 7, device="cuda")
        msteps = args.steps if wl == "mtp_b64_t4" else leg_steps(args.steps, 200)
        mwarm = args.warmup if wl == "mtp_b64_t4" else leg_warm
        sampler_m = ClockSampler(local)
        mms, mlaunch = time_steps(lambda s: mtp_call(gdn, s), msets, msteps, mwarm, world, sampler_m, graph=True)
        mbytes = gdn.workloads.mtp_bytes_per_seq(mt) * mb
        mres = {"workload": "mtp_b64_t4", "gbs": sum_over_ranks(mbytes, world) / (mms * 1e-3) / 1e9,
                "tokens_per_s": sum_over_ranks(mb * mt, world) / (mms * 1e-3), "ms_per_step": mms, "steps": msteps,
                "roofline": {"bound": "hbm", "achieved": mbytes / (mlaunch * 1e-3) / 1e9, "peak": hbm_peak,
                             "unit": "GB/s", "frac": mbytes / (mlaunch * 1e-3) / 1e9 / hbm_peak,
                             "peak_kind": f"{peak_kind} hbm_gbs (copy, burst)", "kernel": "decode_mtp_chunk_kernel",
                             "traffic": profile_traffic("gdn_decode_mtp_b64_t4"),
                             "avg_launch_us": mlaunch * 1e3, "algorithmic_bytes_per_launch": mbytes},
                "clocks": sampler_m.summary()}
        if wl == "mtp_b64_t4":
            # the same call at 1 .. 8 tokens per sequence (T = 1 is the single-token kernel on the
            # indexed slots, 2 .. 8 the chunked kernel)
            sweep = {}
            for tt in range(1, 9):
                tsets = msets if tt == mt else mtp_sets(gdn, mb, tt, 3, seed=rank + 7, device="cuda")
                tms, tlaunch = time_steps(lambda s: mtp_call(gdn, s), tsets, msteps, mwarm, world, None, graph=True)
                tbytes = gdn.workloads.mtp_bytes_per_seq(tt) * mb
                sweep[str(tt)] = {"us_per_call": tlaunch * 1e3, "gbs": tbytes / (tlaunch * 1e-3) / 1e9,
                                  "frac": tbytes / (tlaunch * 1e-3) / 1e9 / hbm_peak}
                if tsets is not msets:
                    del tsets
            mres["tokens_sweep"] = sweep
            result.update(metric="GDN multi-token decode state GB/s", value=mres["gbs"], unit="GB/s",
                          ms_per_step=mms, dtype="f32",
                          config={"workload": wl, "batch_per_rank": mb, "tokens_per_seq": mt,
                                  "pool_slots": 3 * mb, "l2": "3 disjoint slot sets, 805 MB pool",
                                  "parallelism": f"dp{world}"},
                          roofline=mres["roofline"], gpu_launches=msteps, clocks=mres["clocks"], e2e=None,
                          tokens_sweep=sweep)
        else:
            result["mtp"] = mres
        del msets
        torch.cuda.empty_cache()
    if wl == "longctx_1x131072":
        # one 131,072-token sequence (all 32 v-heads): 1 GPU = the prefill with its in-GPU
        # context-parallel segments; N GPUs = context parallelism across ranks (strong scaling:
        # the same sequence split by context_parallel.split_ranges, maps exchanged over NCCL)
        L = 131072
        seqlens = [L]
        inp = gdn.workloads.prefill_inputs(seqlens, seed=11, device="cuda")
        if world == 1:
            inp["output"] = torch.empty(L, 32, 128, dtype=torch.bfloat16, device="cuda")
            inp["new_state"] = torch.empty_like(inp["state"])
            call = lambda s: prefill_call(gdn, s)  # noqa: E731
            local_tokens, launches = L, prefill_launches(gdn, seqlens)
        else:
            loc = gdn.context_parallel.local_inputs(inp, world, rank)
            inp = loc
            cp = gdn.context_parallel

            def call(s):
                cp.prefill_context_parallel(s["q"], s["k"], s["v"], s["state"], s["A_log"], s["a"], s["dt_bias"],
                                            s["b"], s["cu_seqlens"], s["scale"])
            local_tokens = int(loc["q"].shape[0])
            launches = prefill_launches(gdn, [local_tokens]) + (0 if rank == 0 else 3)
        sampler_l = ClockSampler(local)
        lms, llaunch = time_steps(call, [inp], args.steps, args.warmup, world, sampler_l)
        flops = gdn.workloads.prefill_flops_per_token() * L
        result.update(metric="GDN long-context prefill tokens/s", value=L / (lms * 1e-3), unit="tokens/s",
                      ms_per_step=lms, dtype="bf16",
                      config={"workload": wl, "seqlens": seqlens, "tokens_per_rank": local_tokens,
                              "l2": "inputs 2.3 GB, larger than L2",
                              "parallelism": "in-GPU segments" if world == 1 else
                              f"context parallel over {world} ranks (weighted ranges, one all_gather of state maps)"},
                      roofline={"bound": "tensor", "achieved": flops / (lms * 1e-3) / 1e12 / world, "peak": bf16_peak,
                                "unit": "TFLOP/s", "frac": flops / (lms * 1e-3) / 1e12 / world / bf16_peak,
                                "peak_kind": f"{peak_kind} bf16_tflops (burst)",
                                "note": "whole step per GPU (all kernels and collectives), algorithmic FLOPs"},
                      gpu_launches=launches * args.steps, clocks=sampler_l.summary(), e2e=None, scaling="strong")
        del inp
        torch.cuda.empty_cache()
    prefill_legs = []
    if wl.startswith("prefill"):
        prefill_legs.append((wl, args.steps, args.warmup))
    elif legs and args.prefill:
        prefill_legs += [("prefill_varlen16", leg_steps(args.steps, 50), leg_warm),
                         ("prefill_8x32768", leg_steps(args.steps, 20), leg_warm)]
    cpu_seqlens = None
    for wl_p, psteps, pwarm in prefill_legs:
        pres, seqlens = prefill_leg(gdn, wl_p, world, rank, local, psteps, pwarm, peaks)
        if wl_p == "prefill_varlen16":
            cpu_seqlens = seqlens
        if wl.startswith("prefill"):
            result.update(metric="GDN prefill tokens/s", value=pres["tokens_per_s"], unit="tokens/s",
                          ms_per_step=pres["ms_per_step"], dtype="bf16",
                          config={"workload": wl_p, "seqlens_per_rank": seqlens,
                                  "l2": "inputs larger than L2 (2 rotating sets)",
                                  "parallelism": f"dp{world}" + (" (sequences split over the ranks)"
                                                                 if wl_p == "prefill_8x32768" else "")},
                          roofline=pres["roofline"], gpu_launches=pres["gpu_launches_per_step"] * psteps,
                          clocks=pres["clocks"], e2e=None, scaling=pres["scaling"])
            if "qk_l2norm" in pres:
                result["qk_l2norm"] = pres["qk_l2norm"]
        else:
            result["prefill" if wl_p == "prefill_varlen16" else wl_p] = pres
    if rank == 0:
        budget = float(os.environ.get("GDN_BENCH_CPU_BUDGET_S", "8"))
        if world == 1 and budget > 0:
            if wl.startswith("decode"):
                v, sample, cores = cpu_decode_rate(gdn, 64 if wl == "decode_b64" else 1024, budget)
                result["cpu_baseline"] = {"value": v, "unit": "GB/s", "cores": cores, "kind": "port",
                                          "sample": sample}
            elif wl == "mtp_b64_t4":
                v, sample, cores = cpu_mtp_rate(gdn, 64, 4, budget)
                result["cpu_baseline"] = {"value": v, "unit": "GB/s", "cores": cores, "kind": "port",
                                          "sample": sample}
            elif wl.startswith("prefill"):
                v, sample, cores = cpu_prefill_rate(gdn, result["config"]["seqlens_per_rank"], budget)
                result["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                                          "sample": sample}
            if cpu_seqlens is not None and "prefill" in result:
                v, sample, cores = cpu_prefill_rate(gdn, cpu_seqlens, budget)
                result["prefill"]["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                                                     "sample": sample}
            if legs:
                result["cpu_torch_reference"] = cpu_torch_reference(budget)
        if world == 1 and legs and args.reference_triton:
            result["reference_triton"] = reference_triton_leg(gdn, args.steps)
        line = {"metric": result["metric"], "value": result["value"], "unit": result["unit"],
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": result["ms_per_step"], "higher_is_better": True,
                "scaling": result.pop("scaling", "weak"),
                "vs_baseline": None, "dtype": result["dtype"], "data": "synthetic (seeded, BASELINE distributions)",
                **{k: v for k, v in result.items() if k not in ("metric", "value", "unit", "ms_per_step", "dtype")}}
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="decode_b64",
                    choices=["decode_b64", "decode_b1024", "prefill_varlen16", "prefill_8x32768", "mtp_b64_t4",
                             "longctx_1x131072"])
    ap.add_argument("--no-prefill", dest="prefill", action="store_false",
                    help="skip the configs[3] and configs[4] prefill legs of the default line")
    ap.add_argument("--no-legs", dest="legs", action="store_false",
                    help="the headline decode only (no configs[2] / prefill / mtp / CPU / reference legs)")
    ap.add_argument("--no-reference-triton", dest="reference_triton", action="store_false",
                    help="skip timing the reference's Triton kernels on the GPU")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), rank)
        return
    world, rank, local = dist_setup(args.gpus)
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
