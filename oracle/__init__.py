"""CPU oracle for the GDN hot path (test infrastructure only).

Nothing in the shipped library imports this package; only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` do.
``gdn_oracle`` is the numpy restatement used as the parity checker;
``c_oracle`` wraps the C restatement (``gdn_oracle.c``), used as the timed
CPU baseline and cross-checked against the numpy one.
"""
from . import gdn_oracle  # noqa: F401
