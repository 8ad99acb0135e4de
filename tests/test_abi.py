"""CPU-side checks of the C ABI: the library loads, exports every symbol that
include/*.h declares, and rejects bad arguments on the host before touching a GPU."""
import ctypes
import glob
import os
import re

import pytest

from conftest import REPO

from deltagrid_b200 import _lib


def _declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?(?:unsigned\s+int|int|size_t|void|const char\*|char\*)\s*\*?\s*(dg_\w+)\s*\(",
                             src, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    names = _declared_symbols()
    for n in ("dg_dense_forward", "dg_dense_step", "dg_pkm_forward", "dg_pkm_step"):
        assert n in names


@pytest.mark.parametrize("name", _declared_symbols())
def test_library_exports_declared_symbol(name):
    L = _lib.lib()
    assert hasattr(L, name), f"{name} declared in include/ but not exported"


def test_abi_version_and_status_strings():
    L = _lib.lib()
    assert L.dg_abi_version() == 1
    assert L.dg_status_string(0) == b"ok"
    assert b"unsupported" in L.dg_status_string(-2)


def test_host_validation_rejects_without_gpu():
    L = _lib.lib()
    # null pointers and bad sizes are refused on the host: no CUDA call is made
    assert L.dg_dense_forward(0, 1, 1, 4, 8, 8, None, None, None, None, None, 0, None, None, None,
                              None, None, None) == -1
    assert L.dg_dense_forward(7, 1, 1, 4, 8, 8, *([None] * 5), 0, *([None] * 5), None) == -1
    assert L.dg_pkm_forward(2, 1, 1, 4, 0, 16, 8, *([None] * 6), 0, None, None, None, None, None) == -1
    assert L.dg_dense_step(2, 0, 1, 8, 8, None, 0, 0, None, 0, 0, None, 0, 0, None, 0, 0, None, 0, 0, 0,
                           None, None, None, None) == -1
    one = ctypes.c_int32(0)
    assert L.dg_read_device_status(None, 0, ctypes.byref(one), None) == -1


def test_python_shim_rejects_cpu_tensors():
    torch = pytest.importorskip("torch")
    from deltagrid_b200 import hsru_delta_cuda as ext
    x = torch.zeros(1, 1, 4, 8)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        ext.forward(x, x, x, torch.zeros(1, 1, 4), torch.zeros(1, 1, 4, 8), torch.zeros(1, 1, 4, 8),
                    torch.ones(1))
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        ext.pkm_forward(x, torch.zeros(1, 1, 4), x, x, torch.zeros(1, 1, 4, 8, dtype=torch.int64),
                        torch.ones(1), torch.zeros(1, 1, 16, 8))


def test_install_registers_module_name():
    import sys

    import deltagrid_b200
    mod = deltagrid_b200.install()
    import hsru_delta_cuda
    assert sys.modules["hsru_delta_cuda"] is mod
    for fn in ("forward", "step", "backward", "pkm_step", "pkm_forward", "pkm_backward"):
        assert callable(getattr(hsru_delta_cuda, fn))
