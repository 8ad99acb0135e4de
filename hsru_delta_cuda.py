"""``import hsru_delta_cuda`` with the repository root on sys.path resolves here.

Re-exports the drop-in module deltagrid_b200.hsru_delta_cuda under the
reference extension's module name (the name src/ops/_backend.py imports).
"""
from deltagrid_b200.hsru_delta_cuda import *  # noqa: F401,F403
from deltagrid_b200.hsru_delta_cuda import (backward, device_status, forward, pkm_backward,  # noqa: F401
                                            pkm_forward, pkm_step, step)
