"""The reference C++ engine's files on the GPU path.

The engine (src/cpp/engine) keeps a model's weights in a DLG1 file and its
recurrent state in DLGS snapshots.  This module reads both through the C ABI
(``dg_dlg1_layout``, ``dg_dlgs_*``, csrc/engine_files.cpp), keeps every layer's
memory state resident on the GPU, advances it with this package's kernels, and
writes snapshots the engine loads back:

* ``Dlg1``         -- a weights file: header, grid, and every array by name
  (numpy views of the file, no copy);
* ``read_state`` / ``write_state`` -- DLGS snapshots (fp32 for the float engine,
  Q16.16 int32 for the fixed-point engine);
* ``GpuMemoryEngine`` -- the memory tier of an engine model on the GPU: Q16.16
  files run the bit-exact fixed-point kernels (``dg_fxp_dense_forward`` /
  ``dg_fxp_pkm_forward``), fp32 and int8 files the fp32 recurrence
  (``hsru_delta_cuda.forward`` / ``pkm_forward``).  It takes the kernel-level
  per-step inputs the engine's memory layer forms (wk, wq, slot indices, v,
  beta, alpha; deltagrid_fxp.cpp:181-413, deltagrid_math.cpp:174-417) in the
  engine's step-major order [T, H, ...].
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import numpy as np

from . import _lib

PREC_F32, PREC_INT8, PREC_FXP = 0, 1, 2
ENC_F32, ENC_Q8, ENC_Q16 = 0, 1, 2
MAX_AXES = 8


class Dlg1Header(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "magic", "version", "model_type", "precision_mode", "num_layers", "d_model", "num_heads", "kernel_size",
        "thinking_cycles", "input_or_vocab", "output_dim", "forecast_horizon", "num_axes", "top_k",
        "actual_slots", "flags")]


class Dlg1Array(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("layer", ctypes.c_int32), ("axis", ctypes.c_int32),
                ("encoding", ctypes.c_int32), ("scale", ctypes.c_float), ("offset", ctypes.c_int64),
                ("count", ctypes.c_int64)]


class DlgsHeader(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "num_layers", "d_model", "num_heads", "actual_slots", "kernel_size", "step_count")]


def _bind():
    L = _lib.lib()
    P = ctypes.c_void_p
    L.dg_dlg1_layout.argtypes = [ctypes.c_char_p, ctypes.POINTER(Dlg1Header), ctypes.POINTER(ctypes.c_int32),
                                 ctypes.c_int, ctypes.POINTER(Dlg1Array), ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    L.dg_dlgs_read_header.argtypes = [ctypes.c_char_p, ctypes.POINTER(DlgsHeader)]
    L.dg_dlgs_read_layer.argtypes = [ctypes.c_char_p, ctypes.POINTER(DlgsHeader), ctypes.c_int, P, P]
    L.dg_dlgs_write.argtypes = [ctypes.c_char_p, ctypes.POINTER(DlgsHeader), ctypes.POINTER(P), ctypes.POINTER(P)]
    L.dg_dlgs_conv_elems.argtypes = [ctypes.POINTER(DlgsHeader)]
    L.dg_dlgs_conv_elems.restype = ctypes.c_size_t
    L.dg_dlgs_mem_elems.argtypes = [ctypes.POINTER(DlgsHeader)]
    L.dg_dlgs_mem_elems.restype = ctypes.c_size_t
    return L


def _path(p) -> bytes:
    return os.fsencode(os.fspath(p))


@dataclass
class ArrayInfo:
    name: str
    layer: int
    axis: int
    encoding: int
    scale: float
    offset: int
    count: int


class Dlg1:
    """A DLG1 weights file (export_deltagrid_binary.py:77-237), mapped read-only."""

    def __init__(self, path):
        L = _bind()
        self.path = os.fspath(path)
        hdr = Dlg1Header()
        grid = (ctypes.c_int32 * MAX_AXES)()
        n = ctypes.c_int(0)
        _lib.check(L.dg_dlg1_layout(_path(path), ctypes.byref(hdr), grid, MAX_AXES, None, 0, ctypes.byref(n)),
                   f"dg_dlg1_layout({self.path})")
        arr = (Dlg1Array * max(n.value, 1))()
        _lib.check(L.dg_dlg1_layout(_path(path), ctypes.byref(hdr), grid, MAX_AXES, arr, n.value, ctypes.byref(n)),
                   f"dg_dlg1_layout({self.path})")
        self.header = {f: getattr(hdr, f) for f, _ in Dlg1Header._fields_}
        self.grid_dim = [grid[a] for a in range(hdr.num_axes)]
        self.arrays = [ArrayInfo(a.name.decode(), a.layer, a.axis, a.encoding, a.scale, a.offset, a.count)
                       for a in arr[:n.value]]
        self._map = np.memmap(self.path, dtype=np.uint8, mode="r")

    @property
    def head_dim(self) -> int:
        return self.header["d_model"] // self.header["num_heads"]

    @property
    def precision(self) -> int:
        return self.header["precision_mode"]

    def info(self, name: str, layer: int = -1, axis: int = -1) -> ArrayInfo:
        for a in self.arrays:
            if a.name == name and a.layer == layer and a.axis == axis:
                return a
        raise KeyError(f"{name} (layer {layer}, axis {axis}) not in {self.path}")

    def has(self, name: str, layer: int = -1, axis: int = -1) -> bool:
        return any(a.name == name and a.layer == layer and a.axis == axis for a in self.arrays)

    def raw(self, name: str, layer: int = -1, axis: int = -1) -> np.ndarray:
        """The stored elements (float32, int8 or Q16.16 int32), a view of the file."""
        a = self.info(name, layer, axis)
        dt = {ENC_F32: np.float32, ENC_Q8: np.int8, ENC_Q16: np.int32}[a.encoding]
        nbytes = a.count * np.dtype(dt).itemsize
        return self._map[a.offset:a.offset + nbytes].view(dt)

    def value(self, name: str, layer: int = -1, axis: int = -1) -> np.ndarray:
        """The array as the engine computes with it: fp32 (int8 times its scale) or Q16.16 int32."""
        a = self.info(name, layer, axis)
        r = self.raw(name, layer, axis)
        if a.encoding == ENC_Q8:
            return r.astype(np.float32) * np.float32(a.scale)
        return np.array(r)


@dataclass
class EngineState:
    """A DLGS snapshot: per layer the conv window and the memory state [H, slots, Dh]."""
    num_layers: int
    d_model: int
    num_heads: int
    actual_slots: int
    kernel_size: int
    step_count: int
    conv: list = field(default_factory=list)
    mem: list = field(default_factory=list)

    def header(self) -> DlgsHeader:
        return DlgsHeader(self.num_layers, self.d_model, self.num_heads, self.actual_slots, self.kernel_size,
                          self.step_count)


def read_state(path, dtype=np.float32) -> EngineState:
    """Loads a snapshot (dtype float32 for the float engine, int32 for Q16.16)."""
    L = _bind()
    h = DlgsHeader()
    _lib.check(L.dg_dlgs_read_header(_path(path), ctypes.byref(h)), f"dg_dlgs_read_header({path})")
    st = EngineState(h.num_layers, h.d_model, h.num_heads, h.actual_slots, h.kernel_size, h.step_count)
    nc, Dh = L.dg_dlgs_conv_elems(ctypes.byref(h)), h.d_model // h.num_heads
    for layer in range(h.num_layers):
        conv = np.empty(nc, dtype=dtype)
        mem = np.empty((h.num_heads, h.actual_slots, Dh), dtype=dtype)
        _lib.check(L.dg_dlgs_read_layer(_path(path), ctypes.byref(h), layer, conv.ctypes.data, mem.ctypes.data),
                   f"dg_dlgs_read_layer({path}, {layer})")
        st.conv.append(conv)
        st.mem.append(mem)
    return st


def write_state(path, st: EngineState) -> None:
    L = _bind()
    h = st.header()
    conv = [np.ascontiguousarray(c) for c in st.conv]
    mem = [np.ascontiguousarray(m) for m in st.mem]
    for a in conv + mem:
        if a.dtype.itemsize != 4:
            raise ValueError("DLGS states hold 4-byte elements (float32 or Q16.16 int32)")
    cp = (ctypes.c_void_p * max(len(conv), 1))(*[c.ctypes.data for c in conv])
    mp = (ctypes.c_void_p * max(len(mem), 1))(*[m.ctypes.data for m in mem])
    _lib.check(L.dg_dlgs_write(_path(path), ctypes.byref(h), cp, mp), f"dg_dlgs_write({path})")


class GpuMemoryEngine:
    """The memory tier of an engine model, its state resident on one GPU.

    ``weights``: a DLG1 file; ``state``: a DLGS snapshot of the same model, or
    None for the engine's zero state.  ``state[l]`` is layer l's memory state, a
    CUDA tensor [H, slots, Dh] (int32 Q16.16 for fixed-point files, float32
    otherwise).  ``run_layer`` advances one layer over T steps; ``save`` writes a
    snapshot the engine loads (deltagrid_load_state / deltagrid_load_state_fxp),
    with the conv windows carried over unchanged from the loaded snapshot and the
    step count advanced by the steps run.
    """

    def __init__(self, weights, state=None, device="cuda"):
        import torch
        self.torch = torch
        self.model = Dlg1(weights)
        h = self.model.header
        self.fxp = h["precision_mode"] == PREC_FXP
        self.np_dtype = np.int32 if self.fxp else np.float32
        self.device = torch.device(device)
        self.H, self.Dh, self.slots = h["num_heads"], self.model.head_dim, h["actual_slots"]
        self.sparse = h["num_axes"] > 0 and h["top_k"] > 0
        if state is not None:
            snap = read_state(state, self.np_dtype)
            if (snap.num_layers, snap.d_model, snap.num_heads, snap.actual_slots, snap.kernel_size) != (
                    h["num_layers"], h["d_model"], h["num_heads"], h["actual_slots"], h["kernel_size"]):
                raise _lib.DeltaGridError(f"snapshot {state} does not match model {weights}")
        else:
            hist = max(h["kernel_size"] - 1, 1)
            snap = EngineState(h["num_layers"], h["d_model"], h["num_heads"], h["actual_slots"], h["kernel_size"], 0,
                               [np.zeros(h["d_model"] * hist, self.np_dtype) for _ in range(h["num_layers"])],
                               [np.zeros((self.H, self.slots, self.Dh), self.np_dtype)
                                for _ in range(h["num_layers"])])
        self.snapshot = snap
        self.layer_steps = [0] * h["num_layers"]      # steps each layer has been advanced since loading
        tdt = torch.int32 if self.fxp else torch.float32
        self.state = [torch.from_numpy(m).to(self.device, tdt) for m in snap.mem]

    def _lanes(self, x, last):
        """[T, H, last] (engine order) -> contiguous [H, T, last] on the device."""
        t = self.torch.as_tensor(np.asarray(x)).to(self.device)
        return t.reshape(t.shape[0], self.H, last).transpose(0, 1).contiguous()

    def run_layer(self, layer, wk, wq, v, beta, alpha, idx=None):
        """Advances layer `layer` over T steps; returns y [T, H, Dh] (numpy, engine order).

        wk, wq [T, H, A]; idx [T, H, A] slot indices (sparse PKM models); v [T, H*Dh];
        beta, alpha [T, H] -- the values the engine's memory layer forms each step.
        """
        torch = self.torch
        T = np.asarray(v).shape[0]
        A = np.asarray(wk).shape[-1]
        wk_l, wq_l = self._lanes(wk, A), self._lanes(wq, A)
        v_l = self._lanes(v, self.Dh)
        b_l = torch.as_tensor(np.asarray(beta)).to(self.device).reshape(T, self.H).t().contiguous()
        a_l = torch.as_tensor(np.asarray(alpha)).to(self.device).reshape(T, self.H).t().contiguous()
        st = self.state[layer]
        if self.fxp:
            from . import fxp
            if self.sparse:
                y, _ = fxp.pkm_forward(wk_l, wq_l, self._lanes(idx, A).to(torch.int32), v_l, b_l, a_l, st)
            else:
                y, _ = fxp.dense_forward(wk_l, wq_l, v_l, b_l, a_l, st)
        else:
            from . import hsru_delta_cuda as ext
            one = lambda x: x.unsqueeze(0)                                 # noqa: E731  [H, ...] -> [1, H, ...]
            if self.sparse:
                y, _, _ = ext.pkm_forward(one(v_l), one(b_l), one(wk_l), one(wq_l), one(self._lanes(idx, A)).long(),
                                          one(a_l), one(st))
            else:
                y, s_fin, _, _ = ext.forward(one(v_l), one(v_l), one(v_l), one(b_l), one(wk_l), one(wq_l), one(a_l),
                                             one(st))
                st.copy_(s_fin[0])
            y = y[0]
        self.layer_steps[layer] += T
        return y.transpose(0, 1).contiguous().cpu().numpy()

    def save(self, path) -> None:
        """Writes the snapshot: memory states from the GPU, conv windows as loaded, the
        step count advanced by the most steps any layer has run since loading."""
        snap = self.snapshot
        mem = [s.cpu().numpy().astype(self.np_dtype, copy=False) for s in self.state]
        steps = max(self.layer_steps, default=0)
        write_state(path, EngineState(snap.num_layers, snap.d_model, snap.num_heads, snap.actual_slots,
                                      snap.kernel_size, snap.step_count + steps, list(snap.conv), mem))
