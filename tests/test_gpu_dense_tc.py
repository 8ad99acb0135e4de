"""Chunkwise tensor-core dense forward (tcgen05) against the CPU oracle, for both
layouts: state columns on TMEM lanes (algo 2, the default) and state rows on TMEM
lanes (algo 3, the earlier kernel).

The oracle runs the per-step recurrence with an fp32 state on the storage-quantised
inputs (delta_kernel.cu:64-121 semantics).  The chunked kernel evaluates the
same recurrence 64 steps at a time with 16-bit MMA operands and fp32
accumulation; bar: max|a-b|/max|b| <= 1e-3 for y and for the final state with
fp16 storage, 8e-3 with bf16 storage (one bf16 ulp is 2^-8 relative; the products
with an input operand then take bf16 copies of the state and of R').
"""
import pytest
import torch

from conftest import rel_err
from inputs import dense_inputs, to_np32
from oracle import oracle as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from deltagrid_b200 import _lib
    from deltagrid_b200 import hsru_delta_cuda as ext

TC = 2
TC_ROWS = 3
ALGOS = [TC, TC_ROWS]
AUTO_TC = TC           # the tensor-core kernel AUTO picks


def _both(d, save=False, storage=O.F16, algo=TC):
    g = {n: (t.cuda() if t is not None else None) for n, t in d.items()}
    r = ext.forward(g["q"], g["k"], g["v"], g["beta"], g["wk"], g["wq"], g["decay"], g["s_init"], save, algo=algo)
    s0 = to_np32(d["s_init"]) if d["s_init"] is not None else None
    yo, so, eo = O.dense_forward(to_np32(d["v"]), to_np32(d["beta"]), to_np32(d["wk"]), to_np32(d["wq"]),
                                 to_np32(d["decay"]), s0, want_err=True)
    return r, (O.round_to(yo, storage), so, eo)


@pytest.mark.parametrize("S", [128, 256, 384, 512])
@pytest.mark.parametrize("algo", ALGOS)
def test_tc_small(algo, S):
    d = dense_inputs(1, 2, 64, S, 64, torch.float16, seed=S)
    (out, s, _, _), (yo, so, _) = _both(d, algo=algo)
    assert rel_err(out.float().cpu().numpy(), yo) < 1e-3
    assert rel_err(s.float().cpu().numpy(), O.round_to(so, O.F16)) < 1e-3


@pytest.mark.parametrize("T", [1, 63, 65, 200, 1000])
@pytest.mark.parametrize("algo", ALGOS)
def test_tc_ragged_lengths(algo, T):
    d = dense_inputs(2, 2, T, 256, 64, torch.float16, seed=T)
    (out, s, _, _), (yo, so, _) = _both(d, algo=algo)
    assert rel_err(out.float().cpu().numpy(), yo) < 1e-3
    assert rel_err(s.float().cpu().numpy(), O.round_to(so, O.F16)) < 1e-3


@pytest.mark.parametrize("dyn,static_decay", [(True, 1.0), (False, 0.999)])
@pytest.mark.parametrize("algo", ALGOS)
def test_tc_decay_and_initial_state(algo, dyn, static_decay):
    d = dense_inputs(2, 3, 300, 512, 64, torch.float16, dynamic=dyn, seed=7, s_init=True,
                     static_decay=static_decay)
    (out, s, err, sf), (yo, so, eo) = _both(d, save=True, algo=algo)
    assert rel_err(out.float().cpu().numpy(), yo) < 1e-3
    assert rel_err(s.float().cpu().numpy(), O.round_to(so, O.F16)) < 1e-3
    assert rel_err(sf.cpu().numpy(), so) < 1e-3
    assert rel_err(err.cpu().numpy(), eo) < 1e-3


@pytest.mark.parametrize("algo", ALGOS)
def test_tc_cfg2_geometry_prefix(algo):
    # cfg2 (the second BASELINE config): slots 512, Dh 64, fp16, wk = normalize(k P^T), wq = q P^T;
    # full T = 4096 on 4 lanes so the CPU oracle stays quick
    d = dense_inputs(1, 4, 4096, 512, 64, torch.float16, seed=11)
    (out, s, _, _), (yo, so, _) = _both(d, algo=algo)
    assert rel_err(out.float().cpu().numpy(), yo) < 1e-3
    assert rel_err(s.float().cpu().numpy(), O.round_to(so, O.F16)) < 1e-3


def test_tc_layouts_agree():
    d = dense_inputs(2, 4, 700, 512, 64, torch.float16, dynamic=True, seed=5, s_init=True)
    g = {n: (t.cuda() if t is not None else None) for n, t in d.items()}
    a = (g["q"], g["k"], g["v"], g["beta"], g["wk"], g["wq"], g["decay"], g["s_init"])
    o1, s1, _, _ = ext.forward(*a, algo=TC_ROWS)
    o2, s2, _, _ = ext.forward(*a, algo=TC)
    assert rel_err(o2.float().cpu().numpy(), o1.float().cpu().numpy()) < 1e-3
    assert rel_err(s2.float().cpu().numpy(), s1.float().cpu().numpy()) < 1e-3


def test_tc_wait_timeout_flags_status():
    """With the wait budget set to zero every bounded wait in the kernel gives up at once:
    the launch must return (no hung wait), flag DG_DEVCHK_TIMEOUT in the device status
    word, and leave the context usable for the next, normal launch."""
    d = dense_inputs(1, 2, 200, 256, 64, torch.float16, seed=9)
    g = {n: (t.cuda() if t is not None else None) for n, t in d.items()}
    a = (g["q"], g["k"], g["v"], g["beta"], g["wk"], g["wq"], g["decay"])
    ext.device_status()
    old = ext.set_wait_limit(0)
    try:
        ext.forward(*a, algo=TC)
        torch.cuda.synchronize()
    finally:
        ext.set_wait_limit(old)
    assert ext.device_status() & 0x4
    out, s, _, _ = ext.forward(*a, algo=TC)
    torch.cuda.synchronize()
    assert ext.device_status() == 0
    yo, so = O.dense_forward(to_np32(d["v"]), to_np32(d["beta"]), to_np32(d["wk"]), to_np32(d["wq"]),
                             to_np32(d["decay"]))
    assert rel_err(out.float().cpu().numpy(), O.round_to(yo, O.F16)) < 1e-3


def test_tc_matches_sequential_kernel():
    d = dense_inputs(4, 4, 512, 256, 64, torch.float16, dynamic=True, seed=3, s_init=True)
    g = {n: (t.cuda() if t is not None else None) for n, t in d.items()}
    a = (g["q"], g["k"], g["v"], g["beta"], g["wk"], g["wq"], g["decay"], g["s_init"])
    o1, s1, _, _ = ext.forward(*a, algo=_lib.ALGO_SEQUENTIAL)
    o2, s2, _, _ = ext.forward(*a, algo=TC)
    assert rel_err(o2.float().cpu().numpy(), o1.float().cpu().numpy()) < 1e-3
    assert rel_err(s2.float().cpu().numpy(), s1.float().cpu().numpy()) < 1e-3


def test_auto_selects_tc_for_fp16_dh64():
    d = dense_inputs(1, 1, 64, 512, 64, torch.float16, seed=1)
    g = {n: (t.cuda() if t is not None else None) for n, t in d.items()}
    a = (g["q"], g["k"], g["v"], g["beta"], g["wk"], g["wq"], g["decay"])
    o_auto, _, _, _ = ext.forward(*a)
    o_tc, _, _, _ = ext.forward(*a, algo=AUTO_TC)
    assert torch.equal(o_auto, o_tc)
    with pytest.raises(RuntimeError, match="unsupported"):
        ext.forward(*(t.float() for t in a), algo=TC)


BF16_TOL = 8e-3


@pytest.mark.parametrize("S,T,dyn,s_init", [(128, 200, False, False), (256, 1000, True, True),
                                            (512, 333, True, False), (384, 64, False, True),
                                            (256, 1, True, True), (512, 65, False, True),
                                            (256, 2048, False, False)])
@pytest.mark.parametrize("algo", ALGOS)
def test_tc_bf16_against_oracle(algo, S, T, dyn, s_init):
    """bf16 storage.  The default kernel at <= 256 slots carries the state and residual
    operands as bf16 hi + lo pairs: its fp32 final state and fp32 residuals meet the fp16
    bar of 1e-3; the bf16-rounded outputs are held to one bf16 ulp (8e-3).  Elsewhere
    (384 / 512 slots, and the rows-layout kernel) the operand copies are single bf16
    values and every output is held to 8e-3."""
    d = dense_inputs(2, 3, T, S, 64, torch.bfloat16, dynamic=dyn, seed=S + T, s_init=s_init)
    (out, s, err, sf), (yo, so, eo) = _both(d, save=True, storage=O.BF16, algo=algo)
    assert out.dtype == torch.bfloat16
    tight = 1e-3 if (algo == TC and S <= 256) else BF16_TOL
    assert rel_err(out.float().cpu().numpy(), yo) < BF16_TOL
    assert rel_err(s.float().cpu().numpy(), O.round_to(so, O.BF16)) < BF16_TOL
    assert rel_err(sf.cpu().numpy(), so) < tight
    assert rel_err(err.cpu().numpy(), eo) < tight


@pytest.mark.parametrize("algo", ALGOS)
def test_tc_bf16_cfg2_geometry_full_length(algo):
    d = dense_inputs(1, 4, 4096, 512, 64, torch.bfloat16, seed=12)
    (out, s, _, _), (yo, so, _) = _both(d, storage=O.BF16, algo=algo)
    assert rel_err(out.float().cpu().numpy(), yo) < BF16_TOL
    assert rel_err(s.float().cpu().numpy(), O.round_to(so, O.BF16)) < BF16_TOL


def test_auto_selects_tc_for_bf16_dh64():
    d = dense_inputs(2, 2, 128, 256, 64, torch.bfloat16, seed=2)
    g = {n: (t.cuda() if t is not None else None) for n, t in d.items()}
    a = (g["q"], g["k"], g["v"], g["beta"], g["wk"], g["wq"], g["decay"])
    o_auto, _, _, _ = ext.forward(*a)
    o_tc, _, _, _ = ext.forward(*a, algo=AUTO_TC)
    o_seq, _, _, _ = ext.forward(*a, algo=_lib.ALGO_SEQUENTIAL)
    assert torch.equal(o_auto, o_tc)
    assert rel_err(o_tc.float().cpu().numpy(), o_seq.float().cpu().numpy()) < BF16_TOL
