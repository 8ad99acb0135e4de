"""Warp-specialised PKM kernel (producer / tensor-core GEMV / update warps) against
the CPU oracle and against the two other PKM kernels on identical inputs.

Shapes cover full 128-byte row parts (>= 120 lanes) and 64-byte halves (two CTAs
per lane), top-8 and top-4 (A = 64, 16), dynamic decay, a 64-slot grid where
rows recur inside the prefetch window at almost every step, ragged metadata
chunks (T not a multiple of 16), out-of-range indices, and crowded chains in
the hazard table (short ones, and ones long enough to force sync mode).

Over long sequences on tiny grids (every slot rewritten every few steps) all
kernels, this one included, drift from the oracle by one or two fp16 ulps at the
largest state elements (about 1.5e-3 relative at T=512 on 256 slots), because
each summation order rounds differently and the rounded rows are fed back; the
cross-kernel checks therefore use T=128 there, and the long run uses the
128 x 128 grid of the benchmark configuration.
"""
import numpy as np
import pytest
import torch

from conftest import rel_err
from inputs import STORAGE, TOL, pkm_inputs, to_np32
from oracle import oracle as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from deltagrid_b200 import _lib
    from deltagrid_b200 import hsru_delta_cuda as ext

WS = 3
PIPE = 2
ONE = 1


def _oracle(d, dtype):
    out, st = O.pkm_forward(to_np32(d["v"]), to_np32(d["beta"]), to_np32(d["wk"]), to_np32(d["wq"]),
                            d["idx"].numpy(), to_np32(d["decay"]), to_np32(d["state"]), STORAGE[dtype])
    return O.round_to(out, STORAGE[dtype]), st


def _run(d, algo):
    g = {n: t.cuda() for n, t in d.items()}
    ext.device_status(clear=True)
    out, st, _ = ext.pkm_forward_algo(g["v"], g["beta"], g["wk"], g["wq"], g["idx"], g["decay"], g["state"],
                                      False, algo)
    torch.cuda.synchronize()
    return out, st


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("B,H,T,G,K,dyn", [
    (2, 2, 128, 8, 8, False),      # 64 slots, all 64 active: every row recurs every step
    (2, 2, 136, 16, 4, True),      # A = 16, ragged last chunk (136 = 8 * 17)
    (1, 4, 256, 32, 8, True),      # halves (4 lanes)
    (16, 8, 128, 32, 8, False),    # 128 lanes: full rows
])
def test_ws_against_oracle(dtype, B, H, T, G, K, dyn):
    d = pkm_inputs(B, H, T, G, K, 64, dtype, dynamic=dyn, seed=G + K + B + T, s_init_scale=0.2)
    out, st = _run(d, WS)
    assert ext.device_status(clear=True) == 0
    yo, so = _oracle(d, dtype)
    assert rel_err(out.float().cpu().numpy(), yo) < TOL[dtype]
    assert rel_err(st.float().cpu().numpy(), so) < TOL[dtype]


@pytest.mark.parametrize("lanes", [(2, 3), (16, 8)])
def test_ws_matches_other_kernels(lanes):
    B, H = lanes
    d = pkm_inputs(B, H, 128, 16, 8, 64, torch.float16, dynamic=True, seed=5, s_init_scale=0.3)
    o3, s3 = _run(d, WS)
    o2, s2 = _run(d, PIPE)
    o1, s1 = _run(d, ONE)
    for o, s in ((o2, s2), (o1, s1)):
        assert rel_err(o3.float().cpu().numpy(), o.float().cpu().numpy()) < 1e-3
        assert rel_err(s3.float().cpu().numpy(), s.float().cpu().numpy()) < 1e-3


def test_ws_out_of_range_indices_skipped_and_flagged():
    d = pkm_inputs(2, 2, 64, 16, 4, 64, torch.float16, seed=3, s_init_scale=0.2)
    idx = d["idx"].clone()
    idx[0, 1, 5, 3] = 16 * 16          # one past the end
    idx[1, 0, 40, 0] = -7
    d["idx"] = idx
    out, st = _run(d, WS)
    assert ext.device_status(clear=True) & _lib.DEVCHK_INDEX_RANGE
    o1, s1 = _run(d, ONE)
    ext.device_status(clear=True)
    assert rel_err(out.float().cpu().numpy(), o1.float().cpu().numpy()) < 1e-3
    assert rel_err(st.float().cpu().numpy(), s1.float().cpu().numpy()) < 1e-3


def test_ws_long_sequence_benchmark_grid():
    d = pkm_inputs(2, 4, 2048, 128, 8, 64, torch.float16, dynamic=False, seed=21, s_init_scale=0.0)
    out, st = _run(d, WS)
    assert ext.device_status(clear=True) == 0
    yo, so = _oracle(d, torch.float16)
    assert rel_err(out.float().cpu().numpy(), yo) < 1e-3
    assert rel_err(st.float().cpu().numpy(), so) < 1e-3


def _head(x):
    """The kernel's hazard-table chain head of slot x (32-bit xor-shift / multiply mix)."""
    x = np.asarray(x, dtype=np.uint64) & 0xFFFFFFFF
    x ^= x >> 16
    x = (x * 0x85EBCA6B) & 0xFFFFFFFF
    x ^= x >> 13
    x = (x * 0xC2B2AE35) & 0xFFFFFFFF
    x ^= x >> 16
    return (x >> 20).astype(np.int64)


def _crowded_inputs(T, A, total, crowd, period, seed):
    """Every `period`-th step carries `crowd` slots of one chain head; the other
    steps re-touch slots of the previous step so forwarding happens around them."""
    xs_all = np.arange(total, dtype=np.int64)
    hd = _head(xs_all)
    order = np.argsort(hd, kind="stable")
    bounds = np.searchsorted(hd[order], np.arange(4097))
    groups = [order[bounds[k]:bounds[k + 1]] for k in range(4096)]
    groups = [g for g in groups if len(g) >= crowd]
    rs = np.random.RandomState(seed)
    d = pkm_inputs(1, 2, T, int(np.sqrt(total)), int(np.sqrt(A)), 64, torch.float16, seed=seed, s_init_scale=0.1)
    idx = d["idx"].clone()
    for h in range(2):
        for t in range(T):
            if t % period == 0:
                g = groups[rs.randint(len(groups))]
                xs = list(rs.choice(g, crowd, replace=False))
                rest = [x for x in rs.choice(total, A, replace=False) if x not in xs][: A - crowd]
                row = xs + rest
            else:
                prev = idx[0, h, max(t - 1, 0)].tolist()
                row = list(dict.fromkeys(prev[:6] + list(rs.choice(total, A, replace=False))))[:A]
            idx[0, h, t] = torch.tensor(row, dtype=torch.int64)
    d["idx"] = idx
    return d


@pytest.mark.parametrize("crowd,period", [(6, 4), (16, 1)])
def test_ws_crowded_chains_exact(crowd, period):
    # (6, 4): chains of a few writers inside the window; (16, 1): every step puts
    # 16 slots on one chain head, walks exceed 16 hops and the affected steps
    # gather all rows after every earlier update
    d = _crowded_inputs(256, 16, 1 << 16, crowd, period, seed=9)
    out, st = _run(d, WS)
    assert ext.device_status(clear=True) == 0
    yo, so = _oracle(d, torch.float16)
    assert rel_err(out.float().cpu().numpy(), yo) < 1e-3
    assert rel_err(st.float().cpu().numpy(), so) < 1e-3


def test_ws_step_pieces_exact():
    """Long calls run as step pieces (the index pre-pass of the next piece beside the
    recurrence of this one).  Crowded chains cross the piece boundaries; the result
    matches the oracle, and splitting the call in two gives the same bits."""
    d = _crowded_inputs(2048, 64, 1 << 16, 6, 4, seed=13)
    out, st = _run(d, WS)
    assert ext.device_status(clear=True) == 0
    yo, so = _oracle(d, torch.float16)
    assert rel_err(out.float().cpu().numpy(), yo) < 1e-3
    assert rel_err(st.float().cpu().numpy(), so) < 1e-3
    g = {n: t.cuda() for n, t in d.items()}
    ys = []
    state = g["state"].clone()
    for a, b in ((0, 1024), (1024, 2048)):
        y, state, _ = ext.pkm_forward_algo(*(g[n][:, :, a:b].contiguous() for n in ("v", "beta", "wk", "wq", "idx")),
                                           g["decay"], state, False, WS)
        ys.append(y)
    torch.cuda.synchronize()
    assert ext.device_status(clear=True) == 0
    assert torch.equal(torch.cat(ys, dim=2), out) and torch.equal(state, st)


def test_ws_rejects_uncovered_shapes():
    d = pkm_inputs(1, 1, 100, 8, 4, 64, torch.float16, seed=1)      # T % 8 != 0
    with pytest.raises(_lib.DeltaGridError):
        _run(d, WS)
    d = pkm_inputs(1, 1, 64, 8, 4, 64, torch.float32, seed=1)       # fp32 state
    with pytest.raises(_lib.DeltaGridError):
        _run(d, WS)


def test_ws_saved_rows_match_one_step_kernel():
    # the reference layer always calls pkm_forward with save_for_backward=True
    # (src/ops/_autograd.py:132): the gathered rows of every step, [B,H,T,A,Dh]
    d = pkm_inputs(2, 4, 128, 16, 8, 64, torch.float16, dynamic=True, seed=17, s_init_scale=0.3)
    idx = d["idx"].clone()
    idx[1, 2, 7, 5] = -1                                   # an out-of-range row saves zeros
    d["idx"] = idx
    res = {}
    for algo in (WS, ONE):
        g = {n: t.cuda() for n, t in d.items()}
        out, st, saved = ext.pkm_forward_algo(g["v"], g["beta"], g["wk"], g["wq"], g["idx"], g["decay"],
                                              g["state"], True, algo)
        torch.cuda.synchronize()
        ext.device_status(clear=True)
        res[algo] = (out.float().cpu(), st.float().cpu(), saved.float().cpu())
    for a, b in zip(res[WS], res[ONE]):
        assert rel_err(a.numpy(), b.numpy()) < 1e-3
    assert torch.count_nonzero(res[WS][2][1, 2, 7, 5]) == 0


def test_ws_wait_timeout_flags_status():
    """With the wait budget at zero every bounded wait of the warp-specialised kernel gives
    up at once: the launch returns (no hung wait), DG_DEVCHK_TIMEOUT is flagged, and the next
    normal launch on the same context is correct."""
    d = pkm_inputs(1, 2, 128, 16, 8, 64, torch.float16, seed=4)
    ext.device_status(clear=True)
    old = ext.set_wait_limit(0)
    try:
        _run(d, WS)
    finally:
        ext.set_wait_limit(old)
    assert ext.device_status() & 0x4
    out, st = _run(d, WS)
    assert ext.device_status() == 0
    yo, so = _oracle(d, torch.float16)
    assert rel_err(out.float().cpu().numpy(), yo) < TOL[torch.float16]


def test_ws_cfg3_full_length():
    """The cfg3 shape (128 x 128 slots, top-8, fp16 state) at its full T = 8192 on 2 lanes."""
    d = pkm_inputs(1, 2, 8192, 128, 8, 64, torch.float16, dynamic=False, seed=31, s_init_scale=0.0)
    out, st = _run(d, WS)
    assert ext.device_status(clear=True) == 0
    yo, so = _oracle(d, torch.float16)
    assert rel_err(out.float().cpu().numpy(), yo) < 1e-3
    assert rel_err(st.float().cpu().numpy(), so) < 1e-3


def test_cfg4_grid_write_stream_full_length():
    """The cfg4 grid (1024 x 1024 = 1,048,576 slots, 128 MiB of fp16 state per lane) with
    its write stream -- unit keys and values, beta = 1, alpha = 1 -- routed by the GPU
    router from N(0, 1/64) routers, at the full T = 16384 of one launch on 2 lanes, against
    the oracle fed the same routed indices and weights."""
    from deltagrid_b200.route import pkm_route
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(41)
    B, H, T, G, Dh = 1, 2, 16384, 1024, 64
    routers = [torch.randn(G, Dh, generator=g) / Dh ** 0.5 for _ in range(2)]
    k = F.normalize(torch.randn(B, H, T, Dh, generator=g), dim=-1).half()
    v = F.normalize(torch.randn(B, H, T, Dh, generator=g), dim=-1).half()
    wk, wq, idx = pkm_route(k.cuda(), k.cuda(), [r.cuda() for r in routers], [r.cuda() for r in routers], 8)
    d = dict(v=v, beta=torch.ones(B, H, T).half(), wk=wk.cpu(), wq=wq.cpu(), idx=idx.cpu(),
             decay=torch.ones(H).half(), state=torch.zeros(B, H, G * G, Dh).half())
    out, st = _run(d, WS)
    assert ext.device_status(clear=True) == 0
    yo, so = _oracle(d, torch.float16)
    assert rel_err(out.float().cpu().numpy(), yo) < 1e-3
    assert rel_err(st.float().cpu().numpy(), so) < 1e-3
