"""gdn_b200 — B200-native Gated DeltaNet (GDN) decode and prefill operators.

Drop-in for the two entry points of the reference solution
(``solution/triton/kernel_decode.py::run`` and ``kernel_prefill.py::run``):
the same tensors, dtypes, k-last fp32 state layout and value-returning
``(output, new_state)`` contract, computed by hand-written sm_100a CUDA
kernels in ``libgdn_b200.so`` reached through a C ABI (``include/gdn_b200.h``).
``kernel_mtp`` adds the serving form: multi-token decode against a state pool;
``context_parallel`` spreads one prefill of few long sequences over the ranks of a
process group (affine state maps exchanged once); ``harness`` runs flashinfer-bench
workload records (definition + safetensors blobs) through the drop-in ``run``s;
``tvm_binding`` is the TVM-FFI route (a native module over the same C ABI).
There is no CPU or Triton fallback: without the built library on a CUDA
device every operator raises.
"""
from . import workloads  # noqa: F401  (CPU-only helpers, always importable)
from . import sharding  # noqa: F401
from . import kernel_decode, kernel_prefill, kernel_mtp  # noqa: F401
from . import context_parallel  # noqa: F401
from . import harness  # noqa: F401
from . import tvm_binding  # noqa: F401
from ._lib import library, library_path  # noqa: F401

__all__ = ["kernel_decode", "kernel_prefill", "kernel_mtp", "context_parallel", "harness", "workloads", "sharding",
           "tvm_binding", "library", "library_path"]
