"""Dense recurrence on the GPU (through the drop-in module and the C ABI) against
the CPU oracle and the reference goldens.

Tolerance, max|a-b|/max|b| per output: 1e-5 for fp32/fp64 storage, 1e-3 for
fp16, 8e-3 for bf16 (the reference's own bf16 outputs differ
from an fp32 evaluation by up to one bf16 ulp, 2^-8 relative, at the top binade).
"""
import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err
from inputs import STORAGE, TOL, dense_inputs, to_np32
from oracle import oracle as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from deltagrid_b200 import _lib
    from deltagrid_b200 import hsru_delta_cuda as ext


def _run(d, dtype, algo=0, save=False):
    dev = "cuda"
    g = {n: (t.to(dev) if t is not None else None) for n, t in d.items()}
    return ext.forward(g["q"], g["k"], g["v"], g["beta"], g["wk"], g["wq"], g["decay"], g["s_init"],
                       save, algo=algo)


def _oracle(d, dtype):
    s0 = to_np32(d["s_init"]) if d["s_init"] is not None else None
    out, s, err = O.dense_forward(to_np32(d["v"]), to_np32(d["beta"]), to_np32(d["wk"]), to_np32(d["wq"]),
                                  to_np32(d["decay"]), s0, want_err=True)
    code = STORAGE[dtype]
    return O.round_to(out, code), s, O.round_to(s, code), err


@pytest.mark.parametrize("name", ["dense_static_f32.npz", "dense_slotproj_dyn_f32.npz"])
def test_reference_loop_golden(name):
    g = load_golden(name)
    t = {k: torch.from_numpy(g[k]).cuda() for k in ("v", "beta", "wk", "wq", "decay", "s_init")}
    out, s, _, _ = ext.forward(t["v"], t["v"], t["v"], t["beta"], t["wk"], t["wq"], t["decay"], t["s_init"])
    assert rel_err(out.cpu().numpy(), g["y"]) < 1e-5
    assert rel_err(s.cpu().numpy(), g["s_final"]) < 1e-5


def test_cfg1_fp32():
    # cfg1, the first BASELINE config: B=4 H=4 T=512 Dh=64 slots=64, fp32, static decay 1, S0 = 0
    d = dense_inputs(4, 4, 512, 64, 64, torch.float32, seed=0)
    out, s, _, _ = _run(d, torch.float32)
    yo, so, _, _ = _oracle(d, torch.float32)
    assert rel_err(out.cpu().numpy(), yo) < TOL[torch.float32]
    assert rel_err(s.cpu().numpy(), so) < TOL[torch.float32]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("S,Dh", [(8, 32), (16, 64), (32, 32), (64, 64), (128, 64), (256, 64),
                                  (512, 64), (48, 40), (1000, 16)])
def test_sequential_shapes(dtype, S, Dh):
    d = dense_inputs(2, 3, 37, S, Dh, dtype, dynamic=(S % 3 == 0), seed=S + Dh, s_init=True,
                     static_decay=0.999)
    out, s, _, _ = _run(d, dtype, algo=_lib.ALGO_SEQUENTIAL)
    yo, _, so, _ = _oracle(d, dtype)
    assert out.dtype == dtype and s.dtype == dtype
    assert rel_err(out.float().cpu().numpy(), yo) < TOL[dtype]
    assert rel_err(s.float().cpu().numpy(), so) < TOL[dtype]


@pytest.mark.parametrize("B,H,T,S,dyn,s_init", [
    (16, 16, 200, 64, False, False),    # 256 lanes: more CTAs than SMs (64-step chunks), ragged last chunk
    (2, 2, 300, 64, True, True),        # one wave (256-step chunks): per-step decay and s_init across chunks
    (2, 3, 333, 48, True, False),       # padded slots, several chunks
    (1, 2, 300, 1000, False, True),     # padded slots beyond 512, several chunks
])
def test_sequential_chunk_boundaries(B, H, T, S, dyn, s_init):
    """The sequential kernel stages inputs in chunks of up to 256 steps (64 when the grid
    spans more than one wave) and carries the next step's key prediction across the
    chunk boundary: multi-chunk runs on both staging sizes, ragged last chunks,
    per-step decay and an initial state crossing the boundaries, padded slot counts."""
    d = dense_inputs(B, H, T, S, 64, torch.float32, dynamic=dyn, seed=B * H + T + S, s_init=s_init,
                     static_decay=0.999)
    out, s, _, _ = _run(d, torch.float32, algo=_lib.ALGO_SEQUENTIAL)
    yo, so, _, _ = _oracle(d, torch.float32)
    assert rel_err(out.cpu().numpy(), yo) < TOL[torch.float32]
    assert rel_err(s.cpu().numpy(), so) < TOL[torch.float32]


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_save_for_backward_outputs(dtype):
    d = dense_inputs(2, 2, 50, 64, 64, dtype, dynamic=True, seed=5, s_init=True)
    out, s, err, sf = _run(d, dtype, save=True)
    _, s32, _, erro = _oracle(d, dtype)
    assert err.dtype == torch.float32 and sf.dtype == torch.float32
    assert rel_err(err.cpu().numpy(), erro) < 1e-4
    assert rel_err(sf.cpu().numpy(), s32) < 1e-4
    if dtype == torch.float32:
        assert sf.data_ptr() == s.data_ptr()       # the reference returns s_final itself


def test_forward_equals_step_loop():
    # reference test_cuda_parity.py:56-110: forward(kernel) == T x step(kernel)
    d = dense_inputs(2, 4, 24, 64, 64, torch.float32, dynamic=True, seed=9)
    g = {n: (t.cuda() if t is not None else None) for n, t in d.items()}
    out, s_fwd, _, _ = ext.forward(g["q"], g["k"], g["v"], g["beta"], g["wk"], g["wq"], g["decay"])
    s = torch.zeros(2, 4, 64, 64, device="cuda")
    ys = []
    for t in range(24):
        y, s = ext.step(g["q"][:, :, t], g["k"][:, :, t], g["v"][:, :, t], g["beta"][:, :, t],
                        g["wk"][:, :, t], g["wq"][:, :, t], g["decay"][:, :, t], s)
        ys.append(y)
    assert (torch.stack(ys, 2) - out).abs().max().item() < 1e-5
    assert (s - s_fwd).abs().max().item() < 1e-5


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.bfloat16])
@pytest.mark.parametrize("S,Dh", [(64, 64), (256, 64), (512, 64), (100, 48)])
def test_step_strided_and_dynamic(dtype, S, Dh):
    B, H = 3, 5
    d = dense_inputs(B, H, 1, S, Dh, dtype, dynamic=True, seed=S, s_init=True)
    # strided (batch, head) views, last dim contiguous, as the layer passes them
    v = torch.randn(B, 2 * H, Dh).to(dtype).cuda()[:, ::2]
    v.copy_(d["v"][:, :, 0].cuda())
    beta = torch.randn(B, 3 * H).to(dtype).cuda()[:, ::3]
    beta.copy_(d["beta"][:, :, 0].cuda())
    decay = torch.randn(H, B).to(dtype).cuda().t()
    decay.copy_(d["decay"][:, :, 0].cuda())
    wk, wq = d["wk"][:, :, 0].cuda(), d["wq"][:, :, 0].cuda()
    s0 = d["s_init"].cuda()
    y, s1 = ext.step(v, v, v, beta, wk, wq, decay, s0)
    yo, _, so, _ = _oracle(d, dtype)
    assert rel_err(y.float().cpu().numpy(), yo[:, :, 0]) < TOL[dtype]
    assert rel_err(s1.float().cpu().numpy(), so) < TOL[dtype]


def test_step_in_place_via_abi():
    B, H, S, Dh = 2, 2, 128, 64
    d = dense_inputs(B, H, 1, S, Dh, torch.float16, seed=3, s_init=True)
    g = {n: t.cuda() for n, t in d.items()}
    s = g["s_init"].clone()
    out = torch.empty(B, H, Dh, dtype=torch.float16, device="cuda")
    v, wk, wq, beta = g["v"][:, :, 0], g["wk"][:, :, 0], g["wq"][:, :, 0], g["beta"][:, :, 0]
    _lib.call("dg_dense_step", 2, B, H, S, Dh, v.data_ptr(), v.stride(0), v.stride(1),
              beta.data_ptr(), beta.stride(0), beta.stride(1), wk.data_ptr(), wk.stride(0), wk.stride(1),
              wq.data_ptr(), wq.stride(0), wq.stride(1), g["decay"].data_ptr(), 0, 0, 1,
              s.data_ptr(), out.data_ptr(), s.data_ptr(), torch.cuda.current_stream().cuda_stream)
    yo, _, so, _ = _oracle(d, torch.float16)
    assert rel_err(out.float().cpu().numpy(), yo[:, :, 0]) < 1e-3
    assert rel_err(s.float().cpu().numpy(), so) < 1e-3


def test_zero_length_and_errors():
    d = dense_inputs(1, 1, 4, 64, 64, torch.float32)
    g = {n: (t.cuda() if t is not None else None) for n, t in d.items()}
    with pytest.raises(RuntimeError):
        ext.forward(g["q"], g["k"], g["v"].half(), g["beta"], g["wk"], g["wq"], g["decay"])
    with pytest.raises(RuntimeError, match="not implemented"):
        ext.forward(g["q"], g["k"], g["v"].int(), g["beta"], g["wk"], g["wq"], g["decay"])
    z = g["v"][:, :, :0]
    out, s, _, _ = ext.forward(z, z, z, g["beta"][:, :, :0], g["wk"][:, :, :0], g["wq"][:, :, :0],
                               g["decay"], torch.ones(1, 1, 64, 64, device="cuda"))
    assert out.shape == (1, 1, 0, 64)
    assert torch.equal(s, torch.ones_like(s))       # T = 0 returns the initial state


def test_current_stream_is_used():
    d = dense_inputs(2, 2, 64, 64, 64, torch.float16, seed=1)
    g = {n: (t.cuda() if t is not None else None) for n, t in d.items()}
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        out, _, _, _ = ext.forward(g["q"], g["k"], g["v"], g["beta"], g["wk"], g["wq"], g["decay"])
    st.synchronize()
    yo, _, _, _ = _oracle(d, torch.float16)
    assert rel_err(out.float().cpu().numpy(), yo) < 1e-3
