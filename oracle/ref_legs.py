"""Timing legs of the reference's own implementations of the recurrence path --
TEST / BASELINE INFRASTRUCTURE ONLY (bench.py's cpu_baseline leg and its
``--impl reference`` arm).  Nothing here is on the product path.

Legs, each on a bounded sample of a bench workload, each reporting tokens/s of
the recurrence (B*T per second, all H heads of a token):

* ``engine_f32`` -- the reference C++ engine's ``dg_memory_layer_step``
  (src/cpp/engine/src/deltagrid_math.cpp:174-417), compiled from the reference
  sources into oracle/_ref, OpenMP over heads as the engine does (:220-223).
* ``engine_q16`` -- the Q16.16 engine's ``dg_memory_layer_step_fxp``
  (src/cpp/engine/src/deltagrid_fxp.cpp:181-413); that engine has no threading of
  its own, so independent contexts (batch rows) run one per host thread.
  Both engine steps include the layer's qkv/beta projection, out_proj and
  LayerNorm; the same number of projection-only calls is timed beside them and
  subtracted, so the value is the recurrence alone (the raw rate is reported too).
* ``pytorch_loop`` -- the reference layer's own CPU path, ``DeltaGridLayer.forward``
  fed in pieces of fewer than 16 tokens, which run its per-step loop
  (src/modules/memory.py:524-539 dense, :466-487 Sparse Delta-PKM); the layer's
  projections, routing and out_proj are timed separately and subtracted.
* ``pytorch_chunk`` -- ``DeltaGridLayer.chunk_forward`` (memory.py:325-410), the
  chunkwise CPU path the layer takes for 16 tokens or more (dense only).
* ``gpu_kernel`` -- the reference CUDA extension built unmodified from
  src/cpp/binding.cpp + src/cpp/delta_kernel.cu for sm_100a (oracle/_ref,
  ``ref_hsru_delta_cuda``), at the workload's full configuration on this GPU.
"""
from __future__ import annotations

import os
import time

import numpy as np

from . import oracle as O

UNIT = "tokens/s"


def _timed(fn, budget_s: float, min_reps: int = 1):
    """Runs fn until budget_s has passed (at least min_reps times); returns (reps, seconds)."""
    reps = 0
    t0 = time.perf_counter()
    while True:
        fn()
        reps += 1
        dt = time.perf_counter() - t0
        if reps >= min_reps and dt >= budget_s:
            return reps, dt


def _engine_args(w):
    H, Dh = w["H"], w["Dh"]
    if w["kind"] in ("dense", "decode"):
        mode = 0 if w["S"] == Dh else 1
        kw = dict(slots=w["S"]) if mode == 1 else {}
    else:
        mode = 2
        kw = dict(G0=w["G"], G1=w["G"], topk=w["K"])
    return mode, H, Dh, kw


def engine_f32(w, threads: int, budget_s: float = 3.0):
    """The fp32 engine step on `contexts` batch rows, recurrence only."""
    if not O.ref_available():
        return None
    O.set_threads(threads)
    mode, H, Dh, kw = _engine_args(w)
    contexts = 1 if w["kind"] == "pkm" and w["G"] >= 1024 else min(w["B"], 4)
    steps = 8 if w["kind"] in ("dense", "decode") and w["S"] >= 256 else 64
    per_token = w.get("L", 1)            # an LM token passes the recurrence of every layer
    O.ref_f32_time(mode, H, Dh, 2, contexts, **kw)         # warm-up
    tot = proj = 0.0
    n = 0
    t_start = time.perf_counter()
    while time.perf_counter() - t_start < budget_s or n == 0:
        t, p = O.ref_f32_time(mode, H, Dh, steps, contexts, **kw)
        tot += t
        proj += p
        n += 1
    toks = n * contexts * steps / per_token
    return dict(value=toks / max(tot - proj, 1e-12), raw_value=toks / tot, unit=UNIT, cores=threads,
                kind="reference", projection_share=proj / tot,
                sample=f"reference fp32 engine dg_memory_layer_step (deltagrid_math.cpp:174-417), {contexts} "
                       f"context(s) x {H} heads x {steps} steps x {n}, OpenMP over heads on {threads} threads; "
                       f"projection-only calls timed alongside and subtracted")


def engine_q16(w, threads: int, budget_s: float = 3.0):
    """The Q16.16 engine step, contexts spread over the host threads, recurrence only."""
    if not O.ref_available():
        return None
    O.set_threads(threads)
    mode, H, Dh, kw = _engine_args(w)
    contexts = threads if not (w["kind"] == "pkm" and w["G"] >= 1024) else max(1, min(threads, 4))
    steps = 4 if w["kind"] in ("dense", "decode") and w["S"] >= 256 else 32
    per_token = w.get("L", 1)
    O.ref_fxp_time(mode, H, Dh, 1, contexts, **kw)
    tot = proj = 0.0
    n = 0
    t_start = time.perf_counter()
    while time.perf_counter() - t_start < budget_s or n == 0:
        t, p = O.ref_fxp_time(mode, H, Dh, steps, contexts, **kw)
        tot += t
        proj += p
        n += 1
    toks = n * contexts * steps / per_token
    return dict(value=toks / max(tot - proj, 1e-12), raw_value=toks / tot, unit=UNIT, cores=threads,
                kind="reference", projection_share=proj / tot,
                sample=f"reference Q16.16 engine dg_memory_layer_step_fxp (deltagrid_fxp.cpp:181-413), {contexts} "
                       f"contexts (one per thread) x {H} heads x {steps} steps x {n}; projection-only calls "
                       f"timed alongside and subtracted")


def _layer(w, torch):
    from .reference_pkg import load_reference_package
    if load_reference_package() is None:
        return None
    from deltagrid.modules.memory import DeltaGridLayer
    H, Dh = w["H"], w["Dh"]
    torch.manual_seed(0)
    if w["kind"] == "pkm":
        layer = DeltaGridLayer(d_model=H * Dh, num_heads=H, grid_dim=(w["G"], w["G"]), top_k=w["K"])
    else:
        layer = DeltaGridLayer(d_model=H * Dh, num_heads=H, num_slots=w["S"])
    return layer.eval()


def pytorch_loop(w, threads: int, budget_s: float = 3.0):
    """The reference layer's per-step CPU loop (pieces of 15 tokens), recurrence only."""
    import torch
    layer = _layer(w, torch)
    if layer is None:
        return None
    torch.set_num_threads(threads)
    H, Dh = w["H"], w["Dh"]
    d = H * Dh
    rows, piece = 1, 15
    x = torch.randn(rows, piece, d)
    per_token = w.get("L", 1)
    state = None
    if w["kind"] == "pkm":
        state = torch.zeros(rows, H, layer.total_slots, Dh)

    def full():
        with torch.no_grad():
            layer(x, state=state)

    def proj_only():     # the layer's work outside the recurrence on the same piece
        with torch.no_grad():
            packed = layer.proj_qkv_beta(x)
            q, k, _ = packed[:, :, :3 * d].chunk(3, dim=-1)
            q = q.view(rows, piece, H, Dh).transpose(1, 2)
            k = torch.nn.functional.normalize(k.view(rows, piece, H, Dh).transpose(1, 2), p=2, dim=-1)
            if w["kind"] == "pkm":
                layer._route_sparse_pkm(k, q)
            else:
                layer._route_dense(k, q)
            layer.norm(layer.out_proj(torch.zeros(rows, piece, d)))

    full()
    proj_only()
    reps, dt = _timed(full, budget_s)
    preps, pdt = _timed(proj_only, min(1.0, budget_s / 3))
    t_full = dt / reps
    t_proj = pdt / preps
    toks = rows * piece / per_token
    path = "memory.py:466-487 (Sparse Delta-PKM)" if w["kind"] == "pkm" else "memory.py:524-539 (dense)"
    return dict(value=toks / max(t_full - t_proj, 1e-12), raw_value=toks / t_full, unit=UNIT, cores=threads,
                kind="reference", projection_share=t_proj / t_full,
                sample=f"reference DeltaGridLayer.forward on CPU, {rows} row x {piece}-token pieces (the per-step "
                       f"loop, {path}), fp32, torch threads {threads}, x{reps}; the layer's projections, routing "
                       f"and out_proj timed alone and subtracted")


def pytorch_chunk(w, threads: int, budget_s: float = 3.0):
    """DeltaGridLayer.chunk_forward on kernel-level inputs (dense workloads)."""
    if w["kind"] == "pkm":
        return None
    import torch
    layer = _layer(w, torch)
    if layer is None:
        return None
    torch.set_num_threads(threads)
    H, Dh, S = w["H"], w["Dh"], w["S"]
    rows = 1
    T = 256 if S >= 256 else 512
    g = torch.Generator().manual_seed(0)
    v = torch.randn(rows, H, T, Dh, generator=g)
    wk = torch.nn.functional.normalize(torch.randn(rows, H, T, S, generator=g), dim=-1)
    wq = torch.randn(rows, H, T, S, generator=g)
    beta = torch.sigmoid(torch.randn(rows, H, T, 1, generator=g))
    decay = torch.ones(H).view(1, H, 1, 1)
    per_token = w.get("L", 1)

    def run():
        with torch.no_grad():
            layer.chunk_forward(v, beta, wk, wq, decay)

    run()
    reps, dt = _timed(run, budget_s)
    return dict(value=reps * rows * T / per_token / dt, unit=UNIT, cores=threads, kind="reference",
                sample=f"reference DeltaGridLayer.chunk_forward (memory.py:325-410) on CPU, {rows} row x {H} heads "
                       f"x T={T}, slots={S}, fp32, torch threads {threads}, x{reps}")


def gpu_kernel(w, make_inputs, torch, device, steps: int = 3):
    """The reference CUDA extension at the workload's configuration on `device`
    (CUDA events around each call; the PKM state is re-zeroed outside the timing)."""
    from .build_ref_cuda import load_prebuilt
    R = load_prebuilt()
    if R is None:
        return None
    d = make_inputs(w, torch, device, seed=1000)
    stream = torch.cuda.current_stream(device)

    def call():
        if w["kind"] == "decode":
            for lay in d["layers"]:
                y, s = R.step(lay["q"], lay["k"], lay["v"], lay["beta"], lay["wk"], lay["wq"], lay["decay"],
                              lay["state"])
                lay["state"] = s
        elif w["kind"] == "dense":
            for _ in range(w.get("L", 1)):
                R.forward(d["q"], d["k"], d["v"], d["beta"], d["wk"], d["wq"], d["decay"], None, False)
        else:
            R.pkm_forward(d["v"], d["beta"], d["wk"], d["wq"], d["idx"], d["decay"], d["state"], False)

    call()
    torch.cuda.synchronize(device)
    ms = []
    for _ in range(steps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        call()
        b.record(stream)
        torch.cuda.synchronize(device)
        ms.append(a.elapsed_time(b))
        if ms[-1] > 5000:          # a slow kernel: one timed call is sample enough
            break
    m = float(np.median(ms))
    toks = w["B"] * w["T"]
    del d
    torch.cuda.empty_cache()
    return dict(value=toks / (m / 1e3), unit=UNIT, ms_per_step=m, calls=len(ms),
                kernel="reference delta_kernel.cu built unmodified for sm_100a (ref_hsru_delta_cuda): "
                       + ("step (delta_grid_step_* kernels, :223-351)" if w["kind"] == "decode" else
                          "forward (launch_delta_grid_forward, :563-622)" if w["kind"] == "dense" else
                          "pkm_forward (delta_pkm_sequence_forward_kernel, :862-921)"))
