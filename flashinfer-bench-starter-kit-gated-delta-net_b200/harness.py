"""Harness shim: run this library on flashinfer-bench workload records without the
``flashinfer_bench`` package.

The reference measures its solution on the contest dataset (``TraceSet.from_path``,
``scripts/run_local.py:40``): definitions plus workloads whose tensors live in
safetensors blobs.  A workload record, as the reference's recorded traces show it
(``output/*_traces.jsonl``), is a JSON line with

    {"definition": "gdn_decode_qk4_v8_d128_k_last" | "gdn_prefill_qk4_v8_d128_k_last" | ...,
     "workload": {"axes": {...}, "uuid": "...",
                  "inputs": {name: {"type": "safetensors", "path": "./blob/...", "tensor_key": name}
                                  | {"type": "scalar", "value": x}}}, ...}

with ``path`` relative to the dataset root.  ``find_records`` collects the GDN records of
every ``*.jsonl`` under a root (workload files or trace files alike), ``load_inputs``
reads one record's tensors onto a device, ``run_record`` calls ``kernel_decode.run`` or
``kernel_prefill.run`` with them, and ``time_record`` times it the way the reference
driver does (warm-up 3, 100 iterations, CUDA events; ``run_local.py:37``).  Correctness
against the definition's reference is the harness's (or the tests') business: this
module only feeds the operators.  The dataset is not available offline; the tests write
records and blobs of the same shape.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

DECODE_PREFIX = "gdn_decode_"
PREFILL_PREFIX = "gdn_prefill_"
_ARGS = {
    "decode": ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "scale"),
    "prefill": ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens", "scale"),
}


def kind_of(definition: str) -> str:
    """"decode" or "prefill" for a GDN definition name (k-last state layout)."""
    if definition.startswith(DECODE_PREFIX):
        return "decode"
    if definition.startswith(PREFILL_PREFIX):
        return "prefill"
    raise ValueError(f"not a GDN decode/prefill definition: {definition!r}")


def read_records(path) -> list[dict]:
    """The GDN workload records of one JSONL file (lines with "definition" and "workload")."""
    out = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            rec = json.loads(line)
            if not isinstance(rec, dict) or "workload" not in rec or "definition" not in rec:
                continue
            if rec["definition"].startswith((DECODE_PREFIX, PREFILL_PREFIX)):
                out.append(rec)
    return out


def find_records(dataset_root, definition: str | None = None) -> list[dict]:
    """Every GDN record under ``dataset_root`` (recursively, ``*.jsonl``), each once by
    workload uuid, optionally of one definition only."""
    seen, out = set(), []
    for path in sorted(Path(dataset_root).rglob("*.jsonl")):
        for rec in read_records(path):
            if definition and rec["definition"] != definition:
                continue
            key = (rec["definition"], rec["workload"].get("uuid"))
            if key[1] is not None and key in seen:
                continue
            seen.add(key)
            out.append(rec)
    return out


def load_inputs(record: dict, dataset_root, device="cuda") -> dict:
    """The record's inputs as keyword arguments of the operator's ``run`` (tensors on
    ``device``; a missing optional ``state`` or ``scale`` is passed as None)."""
    from safetensors import safe_open

    kind = kind_of(record["definition"])
    root = Path(dataset_root)
    inputs = record["workload"]["inputs"]
    files: dict = {}
    kwargs = {}
    try:
        for name in _ARGS[kind]:
            spec = inputs.get(name)
            if spec is None:
                if name in ("state", "scale"):
                    kwargs[name] = None
                    continue
                raise KeyError(f"workload {record['workload'].get('uuid')} has no input {name!r}")
            if spec["type"] == "scalar":
                kwargs[name] = spec["value"]
            elif spec["type"] == "safetensors":
                path = (root / spec["path"]).resolve()
                if path not in files:
                    files[path] = safe_open(str(path), framework="pt", device="cpu")
                kwargs[name] = files[path].get_tensor(spec.get("tensor_key", name)).to(device)
            else:
                raise ValueError(f"input {name!r}: unsupported type {spec['type']!r}")
    finally:
        files.clear()
    return kwargs


def run_record(record: dict, dataset_root, device="cuda"):
    """Run one workload through this library's drop-in ``run``; returns its
    ``(output, new_state)``."""
    from . import kernel_decode, kernel_prefill

    kw = load_inputs(record, dataset_root, device)
    op = kernel_decode if kind_of(record["definition"]) == "decode" else kernel_prefill
    return op.run(**kw)


def time_record(record: dict, dataset_root, warmup: int = 3, iters: int = 100, device="cuda") -> dict:
    """Mean latency of one workload (inputs resident on the device, CUDA events around
    ``iters`` calls after ``warmup``), as the reference driver measures it."""
    from . import kernel_decode, kernel_prefill

    kw = load_inputs(record, dataset_root, device)
    op = kernel_decode if kind_of(record["definition"]) == "decode" else kernel_prefill
    for _ in range(warmup):
        op.run(**kw)
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        op.run(**kw)
    end.record()
    torch.cuda.synchronize(device)
    return {"definition": record["definition"], "uuid": record["workload"].get("uuid"),
            "axes": record["workload"].get("axes", {}), "latency_ms": start.elapsed_time(end) / iters}
