"""deltagrid_b200 -- B200 (sm_100a) kernels for DeltaGrid's recurrence hot path.

* ``deltagrid_b200.hsru_delta_cuda`` -- drop-in for the reference extension
  module ``hsru_delta_cuda`` (same six functions and signatures);
* ``deltagrid_b200.install()`` -- registers it under that name in sys.modules so
  the reference loader (src/ops/_backend.py) finds it;
* ``deltagrid_b200._lib`` -- the ctypes binding of the C ABI
  (include/deltagrid_b200.h) that both sit on.
"""
from __future__ import annotations

import sys

__all__ = ["install", "hsru_delta_cuda"]


def install() -> object:
    """Make ``import hsru_delta_cuda`` resolve to this package's drop-in module."""
    import importlib
    mod = importlib.import_module(__name__ + ".hsru_delta_cuda")
    sys.modules["hsru_delta_cuda"] = mod
    return mod


def __getattr__(name):
    if name == "hsru_delta_cuda":
        import importlib
        return importlib.import_module(__name__ + ".hsru_delta_cuda")
    raise AttributeError(name)
