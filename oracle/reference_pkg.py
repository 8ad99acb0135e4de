"""Test infrastructure and reference-arm timing only: the reference's own Python package (src/ -- DeltaGridLM,
DeltaGridBlock, DeltaGridLayer), installed from the reference sources into
baseline/_ref (git-ignored), and a switch for the CUDA extension its layers call
(src/ops/_backend.py:21-80 caches one module under the name hsru_delta_cuda).

The installed package's __init__ imports src/cpp/engine/tools/export_deltagrid_binary,
which the reference's setup.py does not package; that one function (a weight
exporter unrelated to the model's forward) is stubbed so the package imports.
"""
from __future__ import annotations

import os
import sys
import types

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SITE = os.path.join(REPO, "baseline", "_ref")


def load_reference_package():
    """The installed reference package `deltagrid`, or None when it is not installed."""
    if not os.path.isfile(os.path.join(REF_SITE, "deltagrid", "__init__.py")):
        return None
    if "deltagrid" in sys.modules:
        return sys.modules["deltagrid"]
    for name in ("deltagrid.cpp", "deltagrid.cpp.engine", "deltagrid.cpp.engine.tools"):
        sys.modules.setdefault(name, types.ModuleType(name))
    stub = types.ModuleType("deltagrid.cpp.engine.tools.export_deltagrid_binary")

    def export_deltagrid_to_bin(*args, **kwargs):
        raise NotImplementedError("weight export is not part of the tested path")

    stub.export_deltagrid_to_bin = export_deltagrid_to_bin
    sys.modules[stub.__name__] = stub
    if REF_SITE not in sys.path:
        sys.path.insert(0, REF_SITE)
    import deltagrid  # noqa: E402
    return deltagrid


def use_backend(module) -> None:
    """Make the reference layers call `module` as their hsru_delta_cuda extension."""
    from deltagrid.ops import _backend
    _backend._CUDA_EXT = module
    _backend._CHECKED = True
