"""CPU oracle for DeltaGrid's recurrence hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
import this module, and only as the checker or as the timed CPU baseline.  The
product (``deltagrid_b200``) never imports it.

It wraps two native libraries with ctypes:

* ``oracle/libdg_oracle.so`` -- the C restatement in ``dg_oracle.c`` (every
  function there cites the reference file:line it follows);
* ``oracle/_ref/libdg_ref_engine.so`` -- the reference's own C++ engine,
  compiled from its sources by ``make -C oracle ref`` and driven by
  ``ref_engine_harness.cpp`` (optional: absent where the reference checkout is
  absent and nothing was prebuilt).

Parity of the restatement is pinned by ``tests/test_oracle_pins.py`` against
golden vectors from the reference PyTorch layer (``tests/golden/``) and against
the reference engine library.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "libdg_oracle.so")
_REF_PATH = os.path.join(HERE, "_ref", "libdg_ref_engine.so")

F32, F64, F16, BF16 = 0, 1, 2, 3

_c_f = ctypes.POINTER(ctypes.c_float)
_c_i32 = ctypes.POINTER(ctypes.c_int32)
_c_i64 = ctypes.POINTER(ctypes.c_int64)

_lib = None
_ref = None


def build(ref: bool = False) -> None:
    """Compile the oracle (and, with ``ref``, the reference engine) via make."""
    subprocess.run(["make", "-C", HERE, "-s", "all"] + (["ref"] if ref else []), check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_round.restype = ctypes.c_float
        L.orc_round.argtypes = [ctypes.c_float, ctypes.c_int]
        L.orc_fxp_mul.restype = ctypes.c_int32
        L.orc_fxp_mul.argtypes = [ctypes.c_int32, ctypes.c_int32]
        L.orc_num_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(_REF_PATH)


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not os.path.exists(_REF_PATH):
            raise FileNotFoundError(
                f"{_REF_PATH} missing: build it with `make -C oracle ref` where the reference checkout exists")
        R = ctypes.CDLL(_REF_PATH)
        R.ref_f32_time.restype = ctypes.c_double
        R.ref_fxp_time.restype = ctypes.c_double
        _ref = R
    return _ref


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_c_f)


def _i32(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_c_i32)


def _i64(a: np.ndarray):
    assert a.dtype == np.int64 and a.flags.c_contiguous
    return a.ctypes.data_as(_c_i64)


def _cf(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def set_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


def round_to(x: np.ndarray, dtype: int) -> np.ndarray:
    """Round fp32 values to a storage dtype (F16 / BF16), returning fp32."""
    y = _cf(x).copy()
    lib().orc_round_array(_f(y), ctypes.c_int64(y.size), dtype)
    return y


def dense_forward(v, beta, wk, wq, decay, s_init=None, dynamic: Optional[bool] = None,
                  want_err: bool = False):
    """Dense recurrence, fp32 state for all T (delta_kernel.cu:64-121).

    Shapes: v [B,H,T,Dh], beta [B,H,T], wk/wq [B,H,T,S], decay [H] or [B,H,T].
    Returns (out [B,H,T,Dh] fp32, s_final [B,H,S,Dh] fp32[, err [B,H,T,Dh]]).
    """
    v, beta, wk, wq, decay = map(_cf, (v, beta, wk, wq, decay))
    B, H, T, Dh = v.shape
    S = wk.shape[-1]
    if dynamic is None:
        dynamic = decay.ndim > 1
    out = np.empty((B, H, T, Dh), np.float32)
    s_final = np.empty((B, H, S, Dh), np.float32)
    err = np.empty((B, H, T, Dh), np.float32) if want_err else None
    s0 = _cf(s_init) if s_init is not None else None
    lib().orc_dense_forward(B, H, T, S, Dh, _f(v), _f(beta), _f(wk), _f(wq), _f(decay),
                            int(bool(dynamic)), _f(s0) if s0 is not None else None,
                            _f(out), _f(s_final), _f(err) if err is not None else None)
    return (out, s_final, err) if want_err else (out, s_final)


def pkm_forward(v, beta, wk, wq, idx, decay, state, state_dtype: int = F32,
                dynamic: Optional[bool] = None, want_saved: bool = False):
    """Sparse PKM recurrence, in place on a copy of ``state`` (delta_kernel.cu:885-920).

    Touched rows are rounded to ``state_dtype`` after every scatter.  Returns
    (out [B,H,T,Dh] fp32 unrounded, new_state fp32[, saved_s_act]).
    """
    v, beta, wk, wq, decay = map(_cf, (v, beta, wk, wq, decay))
    idx = np.ascontiguousarray(np.asarray(idx, dtype=np.int64))
    st = _cf(state).copy()
    B, H, T, Dh = v.shape
    A = wk.shape[-1]
    total = st.shape[2]
    if dynamic is None:
        dynamic = decay.ndim > 1
    out = np.empty((B, H, T, Dh), np.float32)
    saved = np.empty((B, H, T, A, Dh), np.float32) if want_saved else None
    lib().orc_pkm_forward(B, H, T, A, ctypes.c_int64(total), Dh, _f(v), _f(beta), _f(wk), _f(wq),
                          _i64(idx), _f(decay), int(bool(dynamic)), _f(st), state_dtype, _f(out),
                          _f(saved) if saved is not None else None)
    return (out, st, saved) if want_saved else (out, st)


def topk_desc(scores, k: int) -> Tuple[np.ndarray, np.ndarray]:
    s = _cf(scores)
    vals = np.empty(k, np.float32)
    ix = np.empty(k, np.int32)
    lib().orc_topk_desc(_f(s), s.size, k, _f(vals), _i32(ix))
    return vals, ix


def pkm_route(k, q, wk0, wk1, wq0, wq1, top_k: int, q_scale=None):
    """Two-axis product-key router (memory.py:240-289).

    k, q [..., Dh]; router weights [G, Dh].  Returns (wk, wq, idx, margin) with
    leading shape of k and last dim top_k**2; margin is the smallest gap between
    the top_k-th and (top_k+1)-th score over both axes.
    """
    k, q = _cf(k), _cf(q)
    lead = k.shape[:-1]
    Dh = k.shape[-1]
    N = int(np.prod(lead))
    wk0, wk1, wq0, wq1 = map(_cf, (wk0, wk1, wq0, wq1))
    G0, G1 = wk0.shape[0], wk1.shape[0]
    A = top_k * top_k
    wk = np.empty((N, A), np.float32)
    wq = np.empty((N, A), np.float32)
    idx = np.empty((N, A), np.int64)
    margin = np.empty(N, np.float32)
    qs = None
    if q_scale is not None:
        qs = _cf(np.broadcast_to(np.asarray(q_scale, np.float32), lead).reshape(N))
    lib().orc_pkm_route(ctypes.c_int64(N), Dh, G0, G1, top_k, _f(k), _f(q), _f(wk0), _f(wk1),
                        _f(wq0), _f(wq1), _f(qs) if qs is not None else None,
                        _f(wk), _f(wq), _i64(idx), _f(margin))
    shp = lead + (A,)
    return wk.reshape(shp), wq.reshape(shp), idx.reshape(shp), margin.reshape(lead)


def fxp_mul(a: int, b: int) -> int:
    return int(lib().orc_fxp_mul(int(a), int(b)))


def fxp_dense_forward(wk, wq, v, beta, alpha, state):
    """Q16.16 dense recurrence (deltagrid_fxp.cpp:380-405); lanes-first int32 arrays."""
    wk, wq, v, beta, alpha = (np.ascontiguousarray(x, dtype=np.int32) for x in (wk, wq, v, beta, alpha))
    st = np.ascontiguousarray(state, dtype=np.int32).copy()
    L, T, S = wk.shape
    Dh = v.shape[-1]
    y = np.empty((L, T, Dh), np.int32)
    lib().orc_fxp_dense_forward(L, T, S, Dh, _i32(wk), _i32(wq), _i32(v), _i32(beta), _i32(alpha),
                                _i32(st), _i32(y))
    return y, st


def fxp_pkm_forward(wk, wq, idx, v, beta, alpha, state):
    """Q16.16 sparse PKM recurrence (deltagrid_fxp.cpp:298-326); lanes-first int32 arrays."""
    wk, wq, idx, v, beta, alpha = (np.ascontiguousarray(x, dtype=np.int32)
                                   for x in (wk, wq, idx, v, beta, alpha))
    st = np.ascontiguousarray(state, dtype=np.int32).copy()
    L, T, A = wk.shape
    Dh = v.shape[-1]
    total = st.shape[1]
    y = np.empty((L, T, Dh), np.int32)
    lib().orc_fxp_pkm_forward(L, T, A, ctypes.c_int64(total), Dh, _i32(wk), _i32(wq), _i32(idx),
                              _i32(v), _i32(beta), _i32(alpha), _i32(st), _i32(y))
    return y, st


def fxp_pkm_route(k, q, wk0, wk1, wq0, wq1, top_k: int, q_scale: int):
    """Q16.16 router for one head (deltagrid_fxp.cpp:246-296)."""
    k, q, wk0, wk1, wq0, wq1 = (np.ascontiguousarray(x, dtype=np.int32) for x in (k, q, wk0, wk1, wq0, wq1))
    A = top_k * top_k
    wk = np.empty(A, np.int32)
    wq = np.empty(A, np.int32)
    idx = np.empty(A, np.int32)
    lib().orc_fxp_pkm_route(k.size, wk0.shape[0], wk1.shape[0], top_k, _i32(k), _i32(q), _i32(wk0),
                            _i32(wk1), _i32(wq0), _i32(wq1), ctypes.c_int32(q_scale),
                            _i32(wk), _i32(wq), _i32(idx))
    return wk, wq, idx


# --------------------------------------------------------------------------
# reference engine harness (oracle/_ref)
# --------------------------------------------------------------------------

def _engine_dims(mode, H, Dh, slots, G0, G1, topk):
    total = G0 * G1 if mode == 2 else (slots if mode == 1 else Dh)
    A = topk * topk if mode == 2 else total
    return total, A


def ref_f32_layer_run(mode: int, H: int, Dh: int, T: int, seed: int, slots: int = 0,
                      G0: int = 0, G1: int = 0, topk: int = 0, dyn: bool = False, state_init=None):
    """Run the reference fp32 engine step T times; returns a dict of exports."""
    R = ref_lib()
    total, A = _engine_dims(mode, H, Dh, slots, G0, G1, topk)
    D = H * Dh
    out = dict(wk=np.empty((T, H, A), np.float32), wq=np.empty((T, H, A), np.float32),
               idx=np.empty((T, H, A), np.int32), v=np.empty((T, D), np.float32),
               beta=np.empty((T, H), np.float32), alpha=np.empty((T, H), np.float32),
               y=np.empty((T, D), np.float32), state=np.empty((H, total, Dh), np.float32))
    s0 = _cf(state_init) if state_init is not None else None
    rc = R.ref_f32_layer_run(mode, H, Dh, slots, G0, G1, topk, int(dyn), T, ctypes.c_ulonglong(seed),
                             _f(s0) if s0 is not None else None,
                             _f(out["wk"]), _f(out["wq"]), _i32(out["idx"]), _f(out["v"]),
                             _f(out["beta"]), _f(out["alpha"]), _f(out["y"]), _f(out["state"]))
    assert rc == 0
    return out


def ref_fxp_layer_run(mode: int, H: int, Dh: int, T: int, seed: int, slots: int = 0,
                      G0: int = 0, G1: int = 0, topk: int = 0, dyn: bool = False, state_init=None):
    """Run the reference Q16.16 engine step T times; returns a dict of int32 exports."""
    R = ref_lib()
    total, A = _engine_dims(mode, H, Dh, slots, G0, G1, topk)
    D = H * Dh
    z = lambda *s: np.empty(s, np.int32)  # noqa: E731
    out = dict(wk=z(T, H, A), wq=z(T, H, A), idx=z(T, H, A), v=z(T, D), beta=z(T, H),
               alpha=z(T, H), y=z(T, D), state=z(H, total, Dh), k=z(T, D), q=z(T, D))
    s0 = np.ascontiguousarray(state_init, dtype=np.int32) if state_init is not None else None
    rc = R.ref_fxp_layer_run(mode, H, Dh, slots, G0, G1, topk, int(dyn), T, ctypes.c_ulonglong(seed),
                             _i32(s0) if s0 is not None else None,
                             *(_i32(out[n]) for n in ("wk", "wq", "idx", "v", "beta", "alpha", "y",
                                                      "state", "k", "q")))
    assert rc == 0
    return out


def ref_fxp_router_weights(H, Dh, G0, G1, topk, dyn, seed):
    R = ref_lib()
    w = [np.empty((G, Dh), np.int32) for G in (G0, G1, G0, G1)]
    qs = np.empty(H, np.int32)
    R.ref_fxp_router_weights(H, Dh, G0, G1, topk, int(dyn), ctypes.c_ulonglong(seed),
                             *(_i32(x) for x in w), _i32(qs))
    return w, qs


def ref_topk_desc(scores, k):
    R = ref_lib()
    s = _cf(scores)
    vals = np.empty(k, np.float32)
    ix = np.empty(k, np.int32)
    R.ref_topk_desc(_f(s), s.size, k, _f(vals), _i32(ix))
    return vals, ix


def ref_f32_time(mode, H, Dh, steps, contexts, slots=0, G0=0, G1=0, topk=0, dyn=False):
    """Seconds for steps x contexts reference engine steps, and the projection-only share."""
    R = ref_lib()
    proj = ctypes.c_double(0.0)
    t = R.ref_f32_time(mode, H, Dh, slots, G0, G1, topk, int(dyn), steps, contexts, ctypes.byref(proj))
    return float(t), float(proj.value)


def ref_fxp_time(mode, H, Dh, steps, contexts, slots=0, G0=0, G1=0, topk=0, dyn=False):
    """Seconds for steps x contexts Q16.16 engine steps (contexts spread over the host
    threads), and the projection-only share."""
    R = ref_lib()
    proj = ctypes.c_double(0.0)
    t = R.ref_fxp_time(mode, H, Dh, slots, G0, G1, topk, int(dyn), steps, contexts, ctypes.byref(proj))
    return float(t), float(proj.value)
