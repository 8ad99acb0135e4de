"""DeltaGrid recurrence benchmark on B200 -- one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg2] [--impl ours|reference]
                    [--scaling strong|weak]

A step is one call of the hot path over one batch of synthetic input resident
in HBM: the dense sequence forward ``hsru_delta_cuda.forward`` (cfg1/cfg2/cfg5p),
the PKM sequence forward ``pkm_forward`` (cfg3/cfg4) or 12 layers of the decode
``step`` (cfg5).  The default workload is cfg2, the second BASELINE config (dense,
B=32 H=16 T=4096 Dh=64 slots=512, fp16 storage, fp32 accumulation), the
configuration the headline metric is quoted on.  At N = 1 the line also carries
a ``workloads`` record: the same device timing and roofline for cfg1, cfg3,
cfg4, cfg5 and cfg5p; PKM workloads add ``with_routing``, the step timed with its
routing (``pkm_fused_forward``: router, pre-pass, recurrence) and the router alone.

``e2e`` is the step through the public routed entry points (``dense_fused_forward``,
``pkm_fused_forward``) from pinned host inputs k, q, v, beta, with the result read
back, in pieces whose copies overlap the compute of their neighbours (batch rows
for dense, steps for PKM with the state carried in place).

``--workload cfg5lm`` runs the fifth config whole: the reference's DeltaGridLM
(its blocks and LM head, from baseline/_ref) with its recurrence on this drop-in,
prefill 2048 and greedy decode 512 of the batch of 256 (sharded over the ranks).

Multi-GPU (torchrun, one process per GPU): strong scaling by default -- the
workload's global batch is split into contiguous batch shards, one per rank,
with all H heads of a row on its rank (``--scaling weak`` gives every rank the
full batch instead).  No collective touches the data path; the timed region is
bracketed by a barrier and device syncs, and the reported time is the max over
ranks (NCCL all-reduce MAX afterwards).  Inputs exceed L2 (126 MB), so no flush
is needed between iterations.

``cpu_baseline`` is the reference's own fp32 C++ engine (compiled from the
reference sources into oracle/_ref), recurrence only, on all host cores.

``--impl reference`` times the reference's own implementations (rank 0 only):
its fp32 C++ engine on all host cores is the line's value; beside it, named legs
for its Q16.16 engine, its PyTorch per-step loop and chunk_forward on the CPU,
and its own CUDA kernel built for sm_100a on this GPU (oracle/ref_legs.py).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

WORKLOADS = {
    "cfg1": dict(kind="dense", B=4, H=4, T=512, S=64, Dh=64, dtype="float32",
                 desc="dense fp32 B=4 H=4 T=512 Dh=64 slots=64"),
    "cfg2": dict(kind="dense", B=32, H=16, T=4096, S=512, Dh=64, dtype="float16",
                 desc="dense fp16 B=32 H=16 T=4096 Dh=64 slots=512"),
    "cfg3": dict(kind="pkm", B=16, H=8, T=8192, G=128, K=8, Dh=64, dtype="float16",
                 desc="PKM fp16 B=16 H=8 T=8192 Dh=64 grid 128x128 top-8, routed keys"),
    "cfg4": dict(kind="pkm", B=8, H=8, T=16384, G=1024, K=8, Dh=64, dtype="float16", writes=True,
                 desc="PKM fp16 B=8 H=8 T=16384 Dh=64 grid 1024x1024 top-8, write stream (beta=1)"),
    # the fifth BASELINE config (the LM) at its decode shape: one step is one token of a 256-sequence
    # batch through the recurrence of all 12 layers (12 dense decode steps), states resident
    "cfg5": dict(kind="decode", B=256, H=12, T=1, S=256, Dh=64, L=12, dtype="bfloat16",
                 desc="LM decode recurrence: 12 layers x dense step, B=256 H=12 slots=256 Dh=64 bf16"),
    # the same LM's prefill: 2048 tokens of the 256-sequence batch through the recurrence of
    # all 12 layers (12 dense forwards; one layer's inputs serve every layer, the kernel's
    # work does not depend on the values)
    "cfg5p": dict(kind="dense", B=256, H=12, T=2048, S=256, Dh=64, L=12, dtype="bfloat16",
                  desc="LM prefill recurrence: 12 layers x dense forward, B=256 H=12 T=2048 slots=256 Dh=64 bf16"),
}
# the fifth BASELINE config whole: the reference's DeltaGridLM (its blocks, MLPs and LM
# head, from the reference package installed in baseline/_ref) with its recurrence on
# this drop-in (`deltagrid_b200.install()`), prefill then greedy decode, batch sharded
LM_CFG = dict(vocab=32000, d_model=768, layers=12, heads=12, slots=256, prefill=2048, decode=512, batch=256,
              desc="DeltaGridLM 12 layers d_model=768 12 heads slots=256 vocab=32000 bf16: prefill 2048 + "
                   "greedy decode 512 at batch 256")
METRIC = "recurrence tokens/sec"
UNIT = "tokens/s"


def _peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def _algorithmic(w):
    """Algorithmic bytes and flops per launch (one step of the bench)."""
    B, H, T, Dh = w["B"], w["H"], w["T"], w["Dh"]
    e = 4 if w["dtype"] == "float32" else 2
    ht = B * H * T
    if w["kind"] == "dense":
        S, L = w["S"], w.get("L", 1)
        per_ht = (2 * Dh + 2 * S) * e + e              # v, y, wk, wq, beta
        return L * (ht * per_ht + B * H * S * Dh * e), L * ht * 6.0 * S * Dh
    if w["kind"] == "decode":
        S, L = w["S"], w["L"]
        per_lane = 2 * S * Dh * e + 2 * S * e + 2 * Dh * e + 2 * e    # state in+out, wk, wq, v, y, beta, decay
        return L * B * H * per_lane, L * B * H * 6.0 * S * Dh
    A = w["K"] ** 2
    per_ht = 2 * A * Dh * e + 2 * Dh * e + e + 2 * A * e + A * 8    # rows in+out, v, y, beta, wk, wq, idx
    return ht * per_ht, ht * 6.0 * A * Dh


class Clocks:
    """nvidia-smi sampler running during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.samples = []
        if self.proc is None:
            return
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                self.samples.append(f)

    def summary(self):
        if not getattr(self, "samples", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for s in self.samples for n, v in zip(names, s[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def make_inputs(w, torch, device, seed=0):
    """Seeded synthetic inputs with the BASELINE distributions, created on the device."""
    import torch.nn.functional as F
    g = torch.Generator(device=device).manual_seed(seed)
    dt = getattr(torch, w["dtype"])
    B, H, T, Dh = w["B"], w["H"], w["T"], w["Dh"]
    if w["kind"] == "decode":
        # per layer: the step inputs the layer forms (memory.py:544-636) and its resident state
        S, L = w["S"], w["L"]
        gp = torch.Generator().manual_seed(1)
        P = torch.empty(S, Dh)
        torch.nn.init.orthogonal_(P, generator=gp)
        P = P.to(device)
        lay = []
        for _ in range(L):
            k = F.normalize(torch.randn(B, H, Dh, device=device, generator=g), dim=-1)
            q = torch.randn(B, H, Dh, device=device, generator=g)
            lay.append(dict(
                q=q.to(dt), k=k.to(dt), v=torch.randn(B, H, Dh, device=device, generator=g).to(dt),
                beta=torch.sigmoid(torch.randn(B, H, device=device, generator=g)).to(dt),
                wk=F.normalize(k @ P.T, dim=-1).to(dt), wq=(q @ P.T).to(dt),
                decay=(0.99 + 0.01 * torch.sigmoid(torch.randn(B, H, device=device, generator=g))).to(dt),
                state=(0.1 * torch.randn(B, H, S, Dh, device=device, generator=g)).to(dt)))
        return dict(layers=lay)
    if w["kind"] == "dense":
        S = w["S"]
        k = F.normalize(torch.randn(B, H, T, Dh, device=device, generator=g), dim=-1)
        q = torch.randn(B, H, T, Dh, device=device, generator=g)
        v = torch.randn(B, H, T, Dh, device=device, generator=g).to(dt)
        beta = torch.sigmoid(torch.randn(B, H, T, device=device, generator=g)).to(dt)
        P = None
        if S == Dh:
            wk, wq = k.to(dt), q.to(dt)
        else:
            gp = torch.Generator().manual_seed(1)
            P = torch.empty(S, Dh)
            torch.nn.init.orthogonal_(P, generator=gp)
            P = P.to(device)
            wk = F.normalize(k @ P.T, dim=-1).to(dt)
            wq = (q @ P.T).to(dt)
            P = P.to(dt)
        decay = torch.ones(H, device=device, dtype=dt)
        # kr, qr, P: the config's own inputs (keys, queries, slot projection) for the
        # end-to-end leg, which routes them on the device (dense_fused_forward)
        return dict(q=v, k=v, v=v, beta=beta, wk=wk, wq=wq, decay=decay, kr=k.to(dt), qr=q.to(dt), P=P)
    G, K = w["G"], w["K"]
    total = G * G
    # routing as the layer does it (memory.py:240-289), on the GPU: two router axes of
    # G rows ~ N(0, 1/Dh) shared by keys and queries (memory.py:156-159)
    from deltagrid_b200.route import pkm_route
    gr = torch.Generator().manual_seed(seed + 1)
    routers = [(torch.randn(G, Dh, generator=gr) / Dh ** 0.5).to(device) for _ in range(2)]
    k = F.normalize(torch.randn(B, H, T, Dh, device=device, generator=g), dim=-1)
    if w.get("writes"):
        # write stream: random unit keys and values, beta = 1, read-out with the same key
        q = k
        beta = torch.ones(B, H, T, device=device, dtype=dt)
    else:
        q = torch.randn(B, H, T, Dh, device=device, generator=g)
        beta = torch.sigmoid(torch.randn(B, H, T, device=device, generator=g)).to(dt)
    kr = k.to(dt)
    qr = kr if w.get("writes") else q.to(dt)
    wk, wq, idx = pkm_route(kr, qr, routers, routers, K)
    del k, q
    v = F.normalize(torch.randn(B, H, T, Dh, device=device, generator=g), dim=-1).to(dt)
    decay = torch.ones(H, device=device, dtype=dt)
    state = torch.zeros(B, H, total, Dh, device=device, dtype=dt)
    # kr, qr, routers: the config's own inputs for the end-to-end leg, which routes them on
    # the device (pkm_fused_forward)
    return dict(v=v, beta=beta, wk=wk, wq=wq, idx=idx, decay=decay, state=state, kr=kr, qr=qr, routers=routers)


def e2e_pieces(w, override=0):
    """[(start, end)] of the end-to-end leg's pieces: batch rows for dense (a piece's
    compute is one chain of chunks whatever its lanes, so few pieces, the first and the
    last small: B/16 rows each and the middle in four, or one row each below 16 rows),
    steps for PKM (eight even pieces in whole 8-step groups, else four, two, one);
    `override` asks for that many even pieces."""
    if w["kind"] == "dense":
        B = w["B"]
        if override:
            n = next(k for k in (override, 1) if B % k == 0)
            sizes = [B // n] * n
        elif B >= 16:
            edge = B // 16
            mid = B - 2 * edge
            sizes = [edge] + [mid // 4 + (1 if i < mid % 4 else 0) for i in range(4)] + [edge]
        else:
            sizes = [1] * B
        return [(sum(sizes[:i]), sum(sizes[:i + 1])) for i in range(len(sizes))]
    T = w["T"]
    n = next(k for k in ((override,) if override else (8, 4, 2, 1)) if T % (8 * k) == 0)
    return [(i * (T // n), (i + 1) * (T // n)) for i in range(n)]


def _sm_count():
    try:
        import torch
        return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    except Exception:
        return 148


def launches_per_step(w, sms=None):
    """Kernels one step launches: the dense kernel; for 16-bit PKM the hazard pre-pass
    and the recurrence (pkm_hazard_kernel, pkm_ws_kernel), four pieces of each when
    the call is long and the recurrence leaves 8 SMs free (one CTA per lane for 120
    lanes or more, else two: the rule of pkm_ws.cu); for decode one step kernel per
    layer (dense_step_vec_kernel)."""
    if w["kind"] == "decode":
        return w["L"]
    if w["kind"] == "pkm" and w["dtype"] != "float32":
        sms = sms if sms is not None else _sm_count()
        lanes = w["B"] * w["H"]
        ctas = lanes * (1 if lanes >= 120 else 2)
        return 8 if w["T"] >= 1024 and w["T"] % 32 == 0 and ctas + 8 <= sms else 2
    return w.get("L", 1)


def run_step(ext, w, d, algo=0):
    if w["kind"] == "decode":
        ys = []
        for lay in d["layers"]:
            y, s = ext.step(lay["q"], lay["k"], lay["v"], lay["beta"], lay["wk"], lay["wq"], lay["decay"],
                            lay["state"])
            lay["state"] = s
            ys.append(y)
        return [ys[-1]]
    if w["kind"] == "dense":
        kw = dict(algo=algo) if algo else {}
        for _ in range(w.get("L", 1) - 1):         # the LM prefill: every layer's recurrence
            ext.forward(d["q"], d["k"], d["v"], d["beta"], d["wk"], d["wq"], d["decay"], **kw)
        return ext.forward(d["q"], d["k"], d["v"], d["beta"], d["wk"], d["wq"], d["decay"], **kw)
    if algo:
        return ext.pkm_forward_algo(d["v"], d["beta"], d["wk"], d["wq"], d["idx"], d["decay"], d["state"], False, algo)
    return ext.pkm_forward(d["v"], d["beta"], d["wk"], d["wq"], d["idx"], d["decay"], d["state"])


def cpu_baseline_port(w, threads):
    """Oracle port (dg_oracle.c, OpenMP over lanes) on a bounded sample of the workload."""
    import numpy as np
    from oracle import oracle as O
    O.set_threads(threads)
    rs = np.random.RandomState(0)
    H, Dh = w["H"], w["Dh"]
    if w["kind"] in ("dense", "decode"):
        S = w["S"]
        T = 64 if S >= 256 else 512
        Bs = 1
        v = rs.randn(Bs, H, T, Dh).astype(np.float32)
        wk = rs.randn(Bs, H, T, S).astype(np.float32)
        wk /= np.linalg.norm(wk, axis=-1, keepdims=True)
        wq = rs.randn(Bs, H, T, S).astype(np.float32)
        beta = (1 / (1 + np.exp(-rs.randn(Bs, H, T)))).astype(np.float32)
        decay = np.ones(H, np.float32)
        t0 = time.perf_counter()
        reps = 0
        while True:
            O.dense_forward(v, beta, wk, wq, decay)
            reps += 1
            if time.perf_counter() - t0 > 3.0:
                break
        dt = time.perf_counter() - t0
        tok = reps * Bs * T
        if "L" in w:                          # a token of the LM passes the recurrence of L layers
            return dict(value=tok / dt / w["L"], unit=UNIT, cores=threads, kind="port",
                        sample=f"oracle dense_forward, {Bs}x{H} lanes x T={T}, slots={S}, fp32, x{reps}, "
                               f"divided by {w['L']} layers")
        return dict(value=tok / dt, unit=UNIT, cores=threads, kind="port",
                    sample=f"oracle dense_forward, {Bs}x{H} lanes x T={T}, slots={S}, fp32, x{reps}")
    G, K = w["G"], w["K"]
    A = K * K
    total = G * G
    T = 256
    Bs = max(1, min(w["B"], 2))
    L = Bs * H
    idx = np.empty((Bs, H, T, A), np.int64)
    for i in range(L):
        for t in range(T):
            a0 = rs.choice(G, K, replace=False)
            a1 = rs.choice(G, K, replace=False)
            idx.reshape(L, T, A)[i, t] = (a0[:, None] * G + a1[None, :]).ravel()
    v = rs.randn(Bs, H, T, Dh).astype(np.float32)
    wk = np.abs(rs.randn(Bs, H, T, A)).astype(np.float32)
    wk /= np.linalg.norm(wk, axis=-1, keepdims=True)
    wq = rs.randn(Bs, H, T, A).astype(np.float32)
    beta = (1 / (1 + np.exp(-rs.randn(Bs, H, T)))).astype(np.float32)
    decay = np.ones(H, np.float32)
    state = np.zeros((Bs, H, total, Dh), np.float32)
    t0 = time.perf_counter()
    reps = 0
    while True:
        O.pkm_forward(v, beta, wk, wq, idx, decay, state, O.F32)
        reps += 1
        if time.perf_counter() - t0 > 3.0:
            break
    dt = time.perf_counter() - t0
    return dict(value=reps * Bs * T / dt, unit=UNIT, cores=threads, kind="port",
                sample=f"oracle pkm_forward, {Bs}x{H} lanes x T={T}, {total} slots, fp32 state, x{reps}")


def reference_arm(args, w):
    """The reference's own implementations of the path (rank 0 only): the fp32 C++
    engine (recurrence only, all host cores) is the value; the other legs ride along."""
    threads = os.cpu_count() or 1
    # set explicitly: under torchrun OMP_NUM_THREADS arrives as 1
    os.environ["OMP_NUM_THREADS"] = str(threads)
    from oracle import oracle as O
    from oracle import ref_legs as RL
    out = {"metric": METRIC, "unit": UNIT, "higher_is_better": True, "impl": "reference",
           "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "dtype": "f32",
           "data": "synthetic", "config": {"workload": args.workload, **{k: v for k, v in w.items()}},
           "host": {"cores": threads, "cpu": _cpu_model()}}
    base = None
    if O.ref_available():
        O.set_threads(threads)
        vals = []
        for _ in range(max(1, args.steps)):
            base = RL.engine_f32(w, threads, budget_s=0.5)
            vals.append(base["value"])
        base["value"] = statistics.median(vals)
        out.update(value=base["value"], cpu_baseline=base)
    else:
        base = cpu_baseline_port(w, threads)
        out.update(value=base["value"], cpu_baseline=base)
    legs = {}
    for name, fn in (("engine_q16", RL.engine_q16), ("pytorch_loop", RL.pytorch_loop),
                     ("pytorch_chunk", RL.pytorch_chunk)):
        try:
            r = fn(w, threads, budget_s=2.0)
        except Exception as e:          # a leg that cannot run here is reported, not fatal
            r = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
        if r is not None:
            legs[name] = r
    out["cpu_legs"] = legs
    try:
        import torch
        if torch.cuda.is_available():
            dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
            torch.cuda.set_device(dev)
            r = RL.gpu_kernel(w, make_inputs, torch, dev)
            if r is not None:
                out["gpu_reference_kernel"] = r
    except Exception as e:
        out["gpu_reference_kernel"] = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    out["e2e"] = {"value": out["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    out["vs_baseline"] = None
    print(json.dumps(out))


def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _roofline(w, launch_ms, traffic=None):
    hbm, _, peak_src = _peaks()
    bytes_alg, flops_alg = _algorithmic(w)
    achieved = bytes_alg / (launch_ms / 1e3) / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
            "traffic": traffic, "peak_source": peak_src, "algorithmic_bytes_per_launch": bytes_alg,
            "launch_ms": launch_ms, "kernels_timed": launches_per_step(w),
            "tensor_tflops_achieved": flops_alg / (launch_ms / 1e3) / 1e12}


def _sub_workload(name, ext, torch, device, steps=5, warmup=3, algo=0):
    """Device timing and roofline of another workload on this GPU (the `workloads` record)."""
    w = dict(WORKLOADS[name])
    d = make_inputs(w, torch, device, seed=1000)
    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        run_step(ext, w, d, algo)
    torch.cuda.synchronize(device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * steps)]
    with Clocks(device.index) as clk:
        for i in range(steps):
            ev[2 * i].record(stream)
            run_step(ext, w, d, algo)
            ev[2 * i + 1].record(stream)
        torch.cuda.synchronize(device)
    ms = [ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(steps)]
    m = statistics.mean(ms)
    routed = None
    if w["kind"] == "pkm":
        routed = _routed_pkm(w, d, ext, torch, stream, steps)
    del d
    torch.cuda.empty_cache()
    rl = _roofline(w, m)
    rec = {"desc": w["desc"], "ms_per_step": m, "value": w["B"] * w["T"] / (m / 1e3), "unit": UNIT,
           "roofline": {k: rl[k] for k in ("bound", "achieved", "peak", "unit", "frac", "peak_source",
                                              "algorithmic_bytes_per_launch", "kernels_timed")},
           "steps": steps, "clocks": clk.summary()}
    if routed is not None:
        rec["with_routing"] = routed
    return rec


def _routed_pkm(w, d, ext, torch, stream, steps):
    """The PKM step with its routing in the timed region: pkm_fused_forward from the
    device-resident keys, queries and router weights (router_tc_kernel, then the hazard
    pre-pass and pkm_ws_kernel), and the router alone, CUDA events on the stream."""
    from deltagrid_b200.route import pkm_route
    qr = d["kr"] if w.get("writes") else d["qr"]

    def fused():
        return ext.pkm_fused_forward(d["kr"], qr, d["v"], d["beta"], d["routers"], d["routers"], None, d["decay"],
                                     d["state"], top_k=w["K"])

    def route():
        return pkm_route(d["kr"], qr, d["routers"], d["routers"], w["K"])

    out = {}
    for name, fn in (("fused", fused), ("router", route)):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * steps)]
        for i in range(steps):
            ev[2 * i].record(stream)
            fn()
            ev[2 * i + 1].record(stream)
        torch.cuda.synchronize()
        out[name] = statistics.mean(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(steps))
    toks = w["B"] * w["T"]
    return {"ms_per_step": out["fused"], "value": toks / (out["fused"] / 1e3), "unit": UNIT,
            "router_ms": out["router"], "router_ms_per_1M_token_heads": out["router"] * 2 ** 20 / (toks * w["H"]),
            "router_share": out["router"] / out["fused"],
            "path": "pkm_fused_forward: router_tc_kernel -> pkm_hazard_kernel -> pkm_ws_kernel (wk, wq, idx via HBM)"}


def _reference_lm_package():
    """The reference's Python package (DeltaGridLM and its blocks) from baseline/_ref.
    Its __init__ imports a weight-export tool that its setup.py does not install; that
    one name is stubbed (it plays no part in running the model)."""
    import types
    site = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isfile(os.path.join(site, "deltagrid", "__init__.py")):
        return None
    if "deltagrid" not in sys.modules:
        for name in ("deltagrid.cpp", "deltagrid.cpp.engine", "deltagrid.cpp.engine.tools"):
            sys.modules.setdefault(name, types.ModuleType(name))
        stub = types.ModuleType("deltagrid.cpp.engine.tools.export_deltagrid_binary")

        def export_deltagrid_to_bin(*a, **k):
            raise NotImplementedError("weight export is not part of this run")

        stub.export_deltagrid_to_bin = export_deltagrid_to_bin
        sys.modules[stub.__name__] = stub
        if site not in sys.path:
            sys.path.insert(0, site)
    import deltagrid
    return deltagrid


def lm_main(args):
    """cfg5 whole: prefill 2048 random token ids, then 512 greedy decode steps, for this
    rank's share of the batch of 256 (strong scaling; --scaling weak: 256 per rank).
    A step is prefill plus decode; the timed region includes the copy of the token ids
    from pinned host memory and the read back of the last generated tokens.  With
    --impl reference the same model runs on the reference's CUDA extension (built from
    its sources into oracle/_ref) instead of this drop-in."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    c = LM_CFG
    if args.impl == "reference":
        from oracle.build_ref_cuda import load_prebuilt
        ext = load_prebuilt()
        if ext is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "reference CUDA extension not built (oracle/_ref)"}))
            return
        sys.modules["hsru_delta_cuda"] = ext
    else:
        import deltagrid_b200
        ext = deltagrid_b200.install()
    DG = _reference_lm_package()
    if DG is None:
        if rank == 0:
            print(json.dumps({"impl": args.impl, "unavailable": "reference package (baseline/_ref) not installed"}))
        return
    from deltagrid.ops import _backend
    _backend._CUDA_EXT, _backend._CHECKED = ext, True
    torch.manual_seed(0)
    model = DG.DeltaGridLM(vocab_size=c["vocab"], d_model=c["d_model"], num_layers=c["layers"], num_heads=c["heads"],
                           num_slots=c["slots"])
    with torch.no_grad():
        for prm in model.parameters():
            if prm.dim() >= 2:
                prm.normal_(0.0, 0.02)
    model = model.to(device=device, dtype=torch.bfloat16).eval()
    B = c["batch"] // world if args.scaling == "strong" else c["batch"]
    if args.batch > 0:
        B = args.batch
    P, D = (args.seq or c["prefill"]), c["decode"]
    g = torch.Generator().manual_seed(100 + rank)
    ids_host = torch.randint(0, c["vocab"], (B, P), generator=g).pin_memory()
    ids = torch.empty_like(ids_host, device=device)
    out_host = torch.empty((B, 1), dtype=torch.int64, pin_memory=True)
    stream = torch.cuda.current_stream(device)

    def step(evs=None):
        with torch.no_grad():
            if evs:
                evs[0].record(stream)
            ids.copy_(ids_host, non_blocking=True)
            out = model(ids, return_state=True)
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
            states = out.state
            del out
            if evs:
                evs[1].record(stream)
            for i in range(D):
                lg, states = model.step(tok, states=states, seq_offset=P + i)
                tok = lg[:, -1].argmax(-1, keepdim=True)
            out_host.copy_(tok, non_blocking=True)
            if evs:
                evs[2].record(stream)

    for _ in range(max(1, min(args.warmup, 2))):
        step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    steps = max(1, args.steps)
    times = []
    with Clocks(local) as clk:
        for _ in range(steps):
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            step(evs)
            torch.cuda.synchronize(device)
            times.append((evs[0].elapsed_time(evs[1]), evs[1].elapsed_time(evs[2])))
    pre = statistics.mean(t[0] for t in times)
    dec = statistics.mean(t[1] for t in times)
    if world > 1:
        tt = torch.tensor([pre, dec, pre + dec], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        pre, dec, tot = (float(x) for x in tt.tolist())
        dist.barrier()
        dist.destroy_process_group()
    else:
        tot = pre + dec
    if rank != 0:
        return
    Bg = B * world
    toks = Bg * (P + D)
    line = {
        "metric": "LM tokens/sec (prefill + decode)", "value": toks / (tot / 1e3), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": max(1, min(args.warmup, 2)), "ms_per_step": tot, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "bf16", "impl": args.impl,
        "data": "synthetic: uniform random token ids, weights ~ N(0, 0.02) (random init)",
        "config": {"workload": "cfg5lm: " + c["desc"], "global_batch": Bg, "per_gpu_batch": B, "prefill": P,
                   "decode": D, "parallelism": f"dp{world} (batch shards, {args.scaling} scaling)"},
        "prefill": {"ms": pre, "tokens_per_s": Bg * P / (pre / 1e3)},
        "decode": {"ms": dec, "tokens_per_s": Bg * D / (dec / 1e3), "ms_per_token": dec / D},
        "e2e": {"value": toks / (tot / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(ids_host.numel() * 8),
                "d2h_bytes_per_step": int(out_host.numel() * 8)},
        "clocks": clk.summary(),
        "model_code": "reference DeltaGridLM (baseline/_ref) with its recurrence on "
                      + ("the reference CUDA extension" if args.impl == "reference" else "deltagrid_b200"),
    }
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="cfg2", choices=sorted(WORKLOADS) + ["cfg5lm"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--algo", type=int, default=0,
                    help="kernel selector: dense 0 auto, 1 sequential, 2 chunked tcgen05 (state columns on TMEM "
                         "lanes), 3 chunked tcgen05 (state rows on TMEM lanes); "
                         "PKM 0 auto, 1 one step, 2 pipelined, 3 warp-specialised")
    ap.add_argument("--batch", type=int, default=0, help="override the per-GPU batch (small profiling cases)")
    ap.add_argument("--seq", type=int, default=0, help="override the sequence length T (small profiling cases)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-pieces", type=int, default=0,
                    help="pieces of the end-to-end step (dense: batch rows, PKM: steps); 0 picks the default")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-workloads", action="store_true", help="skip the other workloads' record (N = 1)")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="strong: the global batch is split over the ranks; weak: every rank runs the full batch")
    args = ap.parse_args()
    if args.workload == "cfg5lm":
        return lm_main(args)
    args.warmup = max(3, args.warmup)
    w = dict(WORKLOADS[args.workload])
    if args.batch > 0:
        w["B"] = args.batch
        w["desc"] += f" (batch overridden to {args.batch})"
    if args.seq > 0:
        w["T"] = args.seq
        w["desc"] += f" (T overridden to {args.seq})"

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            reference_arm(args, w)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from deltagrid_b200 import hsru_delta_cuda as ext

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    # this rank's batch shard (strong scaling) or the whole batch (weak)
    global_B = w["B"] if args.scaling == "strong" else w["B"] * world
    if args.scaling == "strong" and world > 1:
        from deltagrid_b200.shard import shard_range
        b0, b1 = shard_range(w["B"], world, rank)
        w["B"] = b1 - b0
    d = make_inputs(w, torch, device, seed=1000 + rank)
    stream = torch.cuda.current_stream(device)

    def step():
        nonlocal d
        r = run_step(ext, w, d, args.algo)
        return r

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)

    # device-timed region: K steps, events on the launching stream
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    with Clocks(local) as clk:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for i in range(args.steps):
            ev[2 * i].record(stream)
            step()
            ev[2 * i + 1].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    total_ms = t_start.elapsed_time(t_end)
    per_launch_ms = [ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)]
    if world > 1:
        tt = torch.tensor([total_ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms = float(tt.item())
    ms_per_step = total_ms / args.steps
    tokens_per_step = global_B * w["T"]
    value = tokens_per_step / (ms_per_step / 1e3)

    # end to end through the public API: pinned host inputs in, result out, every step
    e2e = None
    if not args.no_e2e and w["kind"] == "decode":
        # every step: the layers' step inputs from pinned host memory, y of the last layer back
        names = ("q", "k", "v", "beta", "wk", "wq", "decay")
        host = [{n: lay[n].to("cpu").pin_memory() for n in names} for lay in d["layers"]]
        h2d = sum(t.numel() * t.element_size() for hl in host for t in hl.values())
        dev_in = [{n: torch.empty_like(lay[n]) for n in names} for lay in d["layers"]]
        y_host = torch.empty(d["layers"][-1]["v"].shape, dtype=d["layers"][-1]["v"].dtype, pin_memory=True)
        d2h = y_host.numel() * y_host.element_size()

        def e2e_step():
            for lay, hl, dl in zip(d["layers"], host, dev_in):
                for n in names:
                    dl[n].copy_(hl[n], non_blocking=True)
            ys = None
            for lay, dl in zip(d["layers"], dev_in):
                ys, lay["state"] = ext.step(dl["q"], dl["k"], dl["v"], dl["beta"], dl["wk"], dl["wq"],
                                            dl["decay"], lay["state"])
            y_host.copy_(ys, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize(device)
        k2 = max(2, min(args.steps, 5))
        if world > 1:
            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(k2):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize(device)
        e_ms = a.elapsed_time(b) / k2
        if world > 1:
            tt = torch.tensor([e_ms], device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e_ms = float(tt.item())
        e2e = {"value": tokens_per_step / (e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e_ms, "steps": k2}
    elif not args.no_e2e:
        # the config's inputs k, q, v, beta cross PCIe and the routing runs on the device:
        # slot projections (dense_fused_forward) or the product-key router (pkm_fused_forward)
        # (the write stream's queries are its keys: copied once).  The step runs in pieces
        # so that the copy in of piece i+1 and the copy out of piece i-1 (their own streams)
        # overlap piece i's compute; what stays exposed is the first piece's copy in and the
        # last piece's compute and copy out.  Dense by batch rows: a piece's compute is one
        # chain of chunks whatever its lanes, so the pieces are few, the first and the last
        # small (B/16 rows) and the middle four even.  PKM by steps, eight even pieces (the
        # state is carried in place from piece to piece, which is how the recurrence treats
        # consecutive calls anyway: rows are rounded to the storage type every step, so the
        # pieces give the unsplit call's results bit for bit).
        names = ("kr", "v", "beta") if w.get("writes") else ("kr", "qr", "v", "beta")
        bounds = e2e_pieces(w, args.e2e_pieces)
        if w["kind"] == "dense":
            cut = lambda t, i: t[bounds[i][0]:bounds[i][1]]
        else:
            cut = lambda t, i: t[:, :, bounds[i][0]:bounds[i][1]]
        npc = len(bounds)
        # pinned host inputs and device buffers, one contiguous block per piece
        host = {n: [cut(d[n], i).to("cpu").contiguous().pin_memory() for i in range(npc)] for n in names}
        h2d = sum(t.numel() * t.element_size() for ts in host.values() for t in ts)
        dev_in = {n: [torch.empty_like(t, device=device) for t in ts] for n, ts in host.items()}

        def compute(i):
            dd = {n: dev_in[n][i] for n in names}
            if w["kind"] == "dense":
                for _ in range(w.get("L", 1)):
                    o = ext.dense_fused_forward(dd["kr"], dd["qr"], dd["v"], dd["beta"], d["P"], d["P"], None,
                                                d["decay"])
                return o[:2]                      # y and the final state of these lanes
            qr = dd["kr"] if w.get("writes") else dd["qr"]
            return ext.pkm_fused_forward(dd["kr"], qr, dd["v"], dd["beta"], d["routers"], d["routers"], None,
                                         d["decay"], d["state"], top_k=w["K"])[:1]     # y of these steps

        def piece_shape(shape, i):
            # the sizing call's output shapes with piece i's rows (dense, dim 0) or steps (PKM, dim 2)
            dim = 0 if w["kind"] == "dense" else 2
            shape = list(shape)
            shape[dim] = bounds[i][1] - bounds[i][0]
            return shape
        # the first piece's real inputs before the sizing call: PKM carries the state in
        # place, so routing uninitialised keys would leave non-finite rows behind
        for n in names:
            dev_in[n][0].copy_(host[n][0])
        first = compute(0)
        res_host = [[torch.empty(piece_shape(o.shape, i), dtype=o.dtype, pin_memory=True) for o in first]
                    for i in range(npc)]
        d2h = sum(t.numel() * t.element_size() for rs in res_host for t in rs)
        s_h2d, s_d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)

        def e2e_step():
            go = torch.cuda.Event()
            go.record(stream)
            s_h2d.wait_event(go)
            landed = []
            with torch.cuda.stream(s_h2d):
                for i in range(npc):
                    for n in names:
                        dev_in[n][i].copy_(host[n][i], non_blocking=True)
                    e = torch.cuda.Event()
                    e.record(s_h2d)
                    landed.append(e)
            for i in range(npc):
                stream.wait_event(landed[i])
                o = compute(i)
                e = torch.cuda.Event()
                e.record(stream)
                s_d2h.wait_event(e)
                with torch.cuda.stream(s_d2h):
                    for src, dst in zip(o, res_host[i]):
                        src.record_stream(s_d2h)
                        dst.copy_(src, non_blocking=True)
            fin = torch.cuda.Event()
            fin.record(s_d2h)
            stream.wait_event(fin)

        e2e_step()
        torch.cuda.synchronize(device)
        k2 = max(2, min(args.steps, 5))
        if world > 1:
            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(k2):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize(device)
        e_ms = a.elapsed_time(b) / k2
        if world > 1:
            tt = torch.tensor([e_ms], device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e_ms = float(tt.item())
        e2e = {"value": tokens_per_step / (e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e_ms, "steps": k2,
               "pieces": f"{npc} ({'batch rows' if w['kind'] == 'dense' else 'steps'}: "
                         f"{[hi - lo for lo, hi in bounds]})"}

    # verification (outside the timed region): per-rank checksums of the last
    # step's outputs gathered over NCCL; no collective touches the data path
    from deltagrid_b200.shard import checksum
    outs = run_step(ext, w, d, args.algo)
    cs = checksum(outs[0])
    verify = None
    if world > 1:
        all_cs = [torch.zeros_like(cs) for _ in range(world)]
        dist.all_gather(all_cs, cs)
        verify = [[float(x) for x in c.tolist()] for c in all_cs]
        dist.barrier()
        dist.destroy_process_group()
    else:
        verify = [[float(x) for x in cs.tolist()]]
    if rank != 0:
        return

    launch_ms = statistics.mean(per_launch_ms)
    traffic = None
    tr_file = os.path.join(HERE, "profiles", f"traffic_{args.workload}.txt")
    if os.path.exists(tr_file) and w["B"] == WORKLOADS[args.workload]["B"]:
        for line in open(tr_file):
            if line.startswith("dram_bytes_per_launch:"):
                traffic = float(line.split(":")[1])
    roofline = _roofline(w, launch_ms, traffic)
    routed = _routed_pkm(w, d, ext, torch, stream, args.steps) if w["kind"] == "pkm" else None

    del d
    torch.cuda.empty_cache()
    workloads = None
    if world == 1 and not args.no_workloads and args.workload == "cfg2" and args.batch == 0 and args.seq == 0:
        workloads = {}
        for name in ("cfg1", "cfg3", "cfg4", "cfg5", "cfg5p"):
            workloads[name] = _sub_workload(name, ext, torch, device)

    cpu = None
    if not args.no_cpu and world == 1:
        threads = os.cpu_count() or 1
        os.environ["OMP_NUM_THREADS"] = str(threads)
        from oracle import oracle as O
        cpu = None
        if O.ref_available():
            from oracle import ref_legs as RL
            cpu = RL.engine_f32(WORKLOADS[args.workload], threads, budget_s=3.0)
        if cpu is None:
            cpu = cpu_baseline_port(WORKLOADS[args.workload], threads)
        cpu["host_cpu"] = _cpu_model()

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": {"float16": "f16", "float32": "f32", "bfloat16": "bf16"}[w["dtype"]],
        "data": "synthetic (seeded, BASELINE distributions, resident in HBM; inputs > L2, no flush)",
        "config": {"workload": f"{args.workload}: {WORKLOADS[args.workload]['desc']}", "global_batch": global_B,
                   "per_gpu_batch": w["B"], "seq_len": w["T"],
                   "parallelism": f"dp{world} (batch shards, {args.scaling} scaling)",
                   "l2": "inputs larger than L2 (no flush)"},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": args.steps * launches_per_step(w),
        "clocks": clk.summary(),
        "verify": {"output_checksums_per_rank": verify},
    }
    if routed is not None:
        line["with_routing"] = routed
    if workloads is not None:
        line["workloads"] = workloads
    print(json.dumps(line))


if __name__ == "__main__":
    main()
