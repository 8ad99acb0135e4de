"""Generate the engine-file fixtures under tests/golden/engine_files/ from the
reference itself.

Run with ``DELTAGRID_REF`` set to the reference project's root (``oracle/refpath.py``) and
``oracle/_ref/libdg_ref_engine.so`` built
(``make -C oracle ref``):

    python tests/golden/make_engine_files.py

For two one-block continuous models of the reference (src/models/continuous.py)
-- Sparse Delta-PKM on a 16 x 16 grid with top-4 (``pkm``) and dense memory with
a 96-slot projection (``dense``), both with the data-dependent decay -- this
writes:

* ``<model>_<prec>.dlg1``: the model exported by the reference's own exporter
  (src/cpp/engine/tools/export_deltagrid_binary.py), prec in fxp / fp32 (and
  int8 for ``pkm``);
* ``<model>_<prec>_a.dlgs``: the reference engine's snapshot after 24 steps from
  its zero state, written by the engine (deltagrid_save_state[_fxp]);
* ``<model>_<prec>_b.dlgs``: the engine's snapshot after 24 more steps, having
  loaded snapshot a; ``<model>_<prec>_run.npz``: the per-step kernel-level inputs
  of those 24 steps and the engine's read-out y;
* ``<model>_src.npz``: source tensors of the model, for the layout checks.

Everything is seeded; rerunning reproduces the files on the same torch version.
"""
from __future__ import annotations

import ctypes
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "engine_files")
sys.path.insert(0, os.path.join(REPO, "oracle"))
from refpath import reference_root  # noqa: E402

REF = reference_root()
sys.path.insert(0, REF)

from src.models.continuous import DeltaGridContinuous  # noqa: E402  (reference package)

T_RUN = 24
MODELS = {
    "pkm": dict(input_dim=6, output_dim=3, d_model=64, num_layers=1, num_heads=2, grid_dim=(16, 16), top_k=4),
    "dense": dict(input_dim=6, output_dim=3, d_model=64, num_layers=1, num_heads=2, num_slots=96),
}


def _exporter():
    path = os.path.join(REF, "src", "cpp", "engine", "tools", "export_deltagrid_binary.py")
    spec = importlib.util.spec_from_file_location("ref_export_deltagrid_binary", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.export_deltagrid_to_bin


def _engine():
    lib = ctypes.CDLL(os.path.join(REPO, "oracle", "_ref", "libdg_ref_engine.so"))
    P, I, U = ctypes.c_void_p, ctypes.c_int, ctypes.c_ulonglong
    for name in ("ref_fxp_file_run", "ref_f32_file_run"):
        getattr(lib, name).argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, I, U] + [P] * 7
        getattr(lib, name).restype = I
    return lib


def _run(lib, prec, weights, state_in, state_out, H, D, A, seed):
    fx = prec == "fxp"
    dt = np.int32 if fx else np.float32
    ex = dict(wk=np.zeros((T_RUN, H, A), dt), wq=np.zeros((T_RUN, H, A), dt),
              idx=np.zeros((T_RUN, H, A), np.int32), v=np.zeros((T_RUN, D), dt), beta=np.zeros((T_RUN, H), dt),
              alpha=np.zeros((T_RUN, H), dt), y=np.zeros((T_RUN, D), dt))
    fn = lib.ref_fxp_file_run if fx else lib.ref_f32_file_run
    rc = fn(weights.encode(), state_in.encode() if state_in else None, state_out.encode(), T_RUN, seed,
            *[ex[k].ctypes.data for k in ("wk", "wq", "idx", "v", "beta", "alpha", "y")])
    assert rc == 0, (weights, rc)
    return ex


def main():
    os.makedirs(OUT, exist_ok=True)
    export = _exporter()
    lib = _engine()
    for mi, (name, kw) in enumerate(MODELS.items()):
        torch.manual_seed(100 + mi)
        model = DeltaGridContinuous(**kw).eval()
        mem = model.blocks[0].memory
        src = dict(decay=mem.decay.detach().float().numpy().ravel(),
                   q_scale=mem.q_scale.detach().float().numpy().ravel(),
                   proj_qkv_beta=mem.proj_qkv_beta.weight.detach().float().numpy(),
                   input_weight=model.feature_proj.weight.detach().float().numpy())
        if mem.axes_proj_k is not None:
            for a, (pk, pq) in enumerate(zip(mem.axes_proj_k, mem.axes_proj_q)):
                src[f"axes_proj_k{a}"] = pk.weight.detach().float().numpy()
                src[f"axes_proj_q{a}"] = pq.weight.detach().float().numpy()
        if mem.slot_proj_k is not None:
            src["slot_proj_k"] = mem.slot_proj_k.weight.detach().float().numpy()
            src["slot_proj_q"] = mem.slot_proj_q.weight.detach().float().numpy()
        np.savez_compressed(os.path.join(OUT, f"{name}_src.npz"), **src)
        H, D = kw["num_heads"], kw["d_model"]
        A = kw["top_k"] ** 2 if "top_k" in kw else mem.actual_slots
        precs = ("fxp", "fp32", "int8") if name == "pkm" else ("fxp", "fp32")
        for prec in precs:
            w = os.path.join(OUT, f"{name}_{prec}.dlg1")
            export(model, w, mode=prec)
            if prec == "int8":
                continue                       # layout checks only
            sa = os.path.join(OUT, f"{name}_{prec}_a.dlgs")
            sb = os.path.join(OUT, f"{name}_{prec}_b.dlgs")
            _run(lib, prec, w, None, sa, H, D, A, seed=11 + mi)
            ex = _run(lib, prec, w, sa, sb, H, D, A, seed=23 + mi)
            np.savez_compressed(os.path.join(OUT, f"{name}_{prec}_run.npz"), **ex)
            print(name, prec, "ok")


if __name__ == "__main__":
    main()
