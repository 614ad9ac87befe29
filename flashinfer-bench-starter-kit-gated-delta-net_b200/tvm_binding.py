"""TVM-FFI route of the drop-in boundary (the reference's CUDA binding route).

The reference's CUDA solution template binds its kernel through TVM-FFI
(``solution/cuda/binding.py:10-25``: ``register_func("flashinfer.kernel")``; the
harness builds ``kernel.cu::<fn>`` with binding ``"tvm-ffi"``, ``README.md:259-279``)
and calls it in destination-passing style.  ``libgdn_b200_tvm_ffi.so``
(``csrc/gdn_tvm_ffi.cc``, host C++ over the C ABI) exports that form natively:

    gdn_decode (q, k, v, state|None, A_log, a, dt_bias, b, scale|None, output, new_state)
    gdn_prefill(q, k, v, state|None, A_log, a, dt_bias, b, cu_seqlens, scale|None, output, new_state)

Arguments are any DLPack tensors (torch tensors pass straight through); work is
enqueued on the stream TVM-FFI holds for the device, so call inside
``tvm_ffi.use_torch_stream()`` to run on torch's current stream.  ``register()``
also publishes them as global functions (``gdn_b200.decode`` / ``gdn_b200.prefill``)
for callers that look kernels up by name, as the template's ``flashinfer.kernel`` is.
"""
from __future__ import annotations

from pathlib import Path

_HERE = Path(__file__).resolve().parent
MODULE_PATH = _HERE / "libgdn_b200_tvm_ffi.so"
_module = None

GLOBAL_NAMES = {"decode": "gdn_decode", "prefill": "gdn_prefill"}


def module():
    """The loaded ``tvm_ffi.Module`` (raises ``RuntimeError`` if tvm_ffi or the module is missing)."""
    global _module
    if _module is not None:
        return _module
    try:
        import tvm_ffi
    except ImportError as e:  # pragma: no cover - tvm_ffi ships with this image
        raise RuntimeError("gdn_b200: the TVM-FFI route needs the tvm_ffi package") from e
    if not MODULE_PATH.exists():
        raise RuntimeError(f"gdn_b200: {MODULE_PATH} is not built (run build.py or __graft_entry__.build())")
    _module = tvm_ffi.load_module(str(MODULE_PATH))
    return _module


def register(prefix: str = "gdn_b200", override: bool = True) -> dict:
    """Register the module's operators as TVM-FFI global functions ``<prefix>.decode`` and
    ``<prefix>.prefill``; returns ``{global name: function}``."""
    import tvm_ffi

    mod = module()
    out = {}
    for short, symbol in GLOBAL_NAMES.items():
        fn = mod.get_function(symbol)
        name = f"{prefix}.{short}"
        tvm_ffi.register_global_func(name, fn, override=override)
        out[name] = fn
    return out


def decode(*args):
    """``gdn_decode`` of the module (destination-passing; see the module docstring)."""
    return module().get_function("gdn_decode")(*args)


def prefill(*args):
    """``gdn_prefill`` of the module (destination-passing; see the module docstring)."""
    return module().get_function("gdn_prefill")(*args)
