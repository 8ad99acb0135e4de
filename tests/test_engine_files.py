"""The reference C++ engine's files: DLG1 weights and DLGS snapshots.

Fixtures (tests/golden/engine_files/, made by make_engine_files.py): two one-block
reference models exported by the reference exporter, and snapshots written by
the reference engine itself before (a) and after (b) 24 further steps, with the
per-step kernel inputs and read-out of those steps.

CPU: the layout walk against the exporter's source tensors (fp32, int8 and
Q16.16 encodings), the refusal of damaged files, byte-identical snapshot
rewrites, and the oracle replaying the 24 steps from snapshot a to snapshot b.
GPU: the same replay through GpuMemoryEngine, bit-exact for Q16.16 files.
"""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, rel_err
from deltagrid_b200 import _lib
from deltagrid_b200 import engine as E
from oracle import oracle as O

FILES = os.path.join(GOLDEN, "engine_files")
RUNS = [("pkm", "fxp"), ("pkm", "fp32"), ("dense", "fxp"), ("dense", "fp32")]


def _f(name):
    return os.path.join(FILES, name)


def _src(model):
    with np.load(_f(f"{model}_src.npz")) as z:
        return {k: z[k] for k in z.files}


def _run(model, prec):
    with np.load(_f(f"{model}_{prec}_run.npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("model,prec", [("pkm", "fp32"), ("pkm", "fxp"), ("pkm", "int8"), ("dense", "fp32"),
                                        ("dense", "fxp")])
def test_dlg1_layout_matches_exported_tensors(model, prec):
    m = E.Dlg1(_f(f"{model}_{prec}.dlg1"))
    h = m.header
    assert h["magic"] == 0x31474C44 and h["version"] == 1 and h["model_type"] == 0
    assert h["precision_mode"] == {"fp32": E.PREC_F32, "int8": E.PREC_INT8, "fxp": E.PREC_FXP}[prec]
    assert (h["num_layers"], h["d_model"], h["num_heads"]) == (1, 64, 2)
    src = _src(model)
    # arrays tile the file after the header and grid, in load order
    ends = [a.offset + a.count * {E.ENC_F32: 4, E.ENC_Q8: 1, E.ENC_Q16: 4}[a.encoding] for a in m.arrays]
    assert ends[-1] == os.path.getsize(m.path)
    vec = {"fp32": lambda x: x.astype(np.float32), "int8": lambda x: x.astype(np.float32),
           "fxp": lambda x: np.round(x.astype(np.float32) * 65536.0).astype(np.int32)}[prec]
    for name, key in (("memory.decay", "decay"), ("memory.q_scale", "q_scale")):
        np.testing.assert_array_equal(m.raw(name, 0), vec(src[key]))
    if model == "pkm":
        assert m.grid_dim == [16, 16] and h["top_k"] == 4 and h["actual_slots"] == 256
        for a in range(2):
            np.testing.assert_array_equal(m.raw("memory.axes_proj_k", 0, a), vec(src[f"axes_proj_k{a}"]).ravel())
            np.testing.assert_array_equal(m.raw("memory.axes_proj_q", 0, a), vec(src[f"axes_proj_q{a}"]).ravel())
    else:
        assert m.grid_dim == [] and h["actual_slots"] == 96 and h["flags"] & 2
        np.testing.assert_array_equal(m.raw("memory.slot_proj_k", 0), vec(src["slot_proj_k"]).ravel())
    w = src["proj_qkv_beta"].astype(np.float32).ravel()
    info = m.info("memory.proj_qkv_beta", 0)
    if prec == "int8":
        # symmetric int8 with the scale stored before the bytes (export_deltagrid_binary.py:60-69)
        scale = np.float32(np.abs(w).max() / 127.0)
        assert info.encoding == E.ENC_Q8 and np.float32(info.scale) == scale
        np.testing.assert_array_equal(m.raw("memory.proj_qkv_beta", 0),
                                      np.clip(np.round(w / scale), -127, 127).astype(np.int8))
        assert rel_err(m.value("memory.proj_qkv_beta", 0), w) < 1e-2
    else:
        np.testing.assert_array_equal(m.raw("memory.proj_qkv_beta", 0), vec(w))


def test_dlg1_refuses_damaged_files(tmp_path):
    good = _f("pkm_fp32.dlg1")
    data = open(good, "rb").read()
    cases = {"truncated": data[:-4], "trailing": data + b"\0\0\0\0", "magic": b"XLG1" + data[4:],
             "precision": data[:12] + (7).to_bytes(4, "little") + data[16:]}
    for name, blob in cases.items():
        p = tmp_path / f"{name}.dlg1"
        p.write_bytes(blob)
        with pytest.raises(_lib.DeltaGridError, match="engine file"):
            E.Dlg1(p)


@pytest.mark.parametrize("model,prec", RUNS)
def test_dlgs_rewrite_is_byte_identical(model, prec, tmp_path):
    for snap in ("a", "b"):
        src = _f(f"{model}_{prec}_{snap}.dlgs")
        st = E.read_state(src, np.int32 if prec == "fxp" else np.float32)
        H, Dh = st.num_heads, st.d_model // st.num_heads
        assert st.mem[0].shape == (H, st.actual_slots, Dh) and st.conv[0].size == st.d_model * 3
        out = tmp_path / f"{snap}.dlgs"
        E.write_state(out, st)
        assert out.read_bytes() == open(src, "rb").read()
    a = E.read_state(_f(f"{model}_{prec}_a.dlgs"))
    b = E.read_state(_f(f"{model}_{prec}_b.dlgs"))
    assert (a.step_count, b.step_count) == (24, 48)


def test_dlgs_refuses_wrong_shape(tmp_path):
    p = tmp_path / "short.dlgs"
    p.write_bytes(open(_f("pkm_fp32_a.dlgs"), "rb").read()[:-8])
    with pytest.raises(_lib.DeltaGridError):
        E.read_state(p)
    with pytest.raises(_lib.DeltaGridError):           # a dense snapshot for the PKM model
        E.GpuMemoryEngine(_f("pkm_fp32.dlg1"), _f("dense_fp32_a.dlgs"), device="cpu")


def _lanes(x, H):
    T = x.shape[0]
    return np.ascontiguousarray(x.reshape(T, H, -1).transpose(1, 0, 2))


@pytest.mark.parametrize("model,prec", RUNS)
def test_oracle_replays_engine_snapshots(model, prec):
    """Snapshot a + the engine's 24 steps of kernel inputs -> snapshot b (oracle, CPU)."""
    fx = prec == "fxp"
    a = E.read_state(_f(f"{model}_{prec}_a.dlgs"), np.int32 if fx else np.float32)
    b = E.read_state(_f(f"{model}_{prec}_b.dlgs"), np.int32 if fx else np.float32)
    r = _run(model, prec)
    H = a.num_heads
    wk, wq, v = _lanes(r["wk"], H), _lanes(r["wq"], H), _lanes(r["v"], H)
    beta, alpha = r["beta"].T.copy(), r["alpha"].T.copy()
    if fx:
        if model == "pkm":
            y, s = O.fxp_pkm_forward(wk, wq, _lanes(r["idx"], H), v, beta, alpha, a.mem[0])
        else:
            y, s = O.fxp_dense_forward(wk, wq, v, beta, alpha, a.mem[0])
        np.testing.assert_array_equal(y, _lanes(r["y"], H))
        np.testing.assert_array_equal(s, b.mem[0])
    else:
        one = lambda x: x[None]                                           # noqa: E731
        if model == "pkm":
            y, s = O.pkm_forward(one(v), one(beta), one(wk), one(wq), one(_lanes(r["idx"], H)).astype(np.int64),
                                 one(alpha), one(a.mem[0]))
        else:
            y, s = O.dense_forward(one(v), one(beta), one(wk), one(wq), one(alpha), s_init=one(a.mem[0]))
        assert rel_err(y[0], _lanes(r["y"], H)) < 1e-5
        assert rel_err(s[0], b.mem[0]) < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("model,prec", RUNS)
def test_gpu_engine_replays_engine_snapshots(model, prec, tmp_path):
    """GpuMemoryEngine: weights + snapshot a on the GPU, the engine's 24 steps, snapshot b."""
    fx = prec == "fxp"
    eng = E.GpuMemoryEngine(_f(f"{model}_{prec}.dlg1"), _f(f"{model}_{prec}_a.dlgs"), "cuda")
    r = _run(model, prec)
    y = eng.run_layer(0, r["wk"], r["wq"], r["v"], r["beta"], r["alpha"], idx=r["idx"] if model == "pkm" else None)
    torch.cuda.synchronize()
    out = tmp_path / "b.dlgs"
    eng.save(out)
    got = E.read_state(out, np.int32 if fx else np.float32)
    ref = E.read_state(_f(f"{model}_{prec}_b.dlgs"), np.int32 if fx else np.float32)
    assert got.step_count == ref.step_count == 48
    yr = r["y"].reshape(y.shape)
    if fx:
        np.testing.assert_array_equal(y, yr)
        np.testing.assert_array_equal(got.mem[0], ref.mem[0])
    else:
        assert rel_err(y, yr) < 1e-5
        assert rel_err(got.mem[0], ref.mem[0]) < 1e-5
    # the conv windows are not advanced by the memory tier: carried from snapshot a
    np.testing.assert_array_equal(got.conv[0], E.read_state(_f(f"{model}_{prec}_a.dlgs"),
                                                            np.int32 if fx else np.float32).conv[0])
