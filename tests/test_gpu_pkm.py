"""Sparse Delta-PKM recurrence on the GPU against the CPU oracle and the reference goldens.

The oracle rounds touched rows to the storage dtype after every step, as the
reference kernel stores them every step (delta_kernel.cu:918).  Tolerance,
max|a-b|/max|b|: 1e-5 for fp32, 1e-3 for fp16, 8e-3 for bf16.
"""
import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err
from inputs import STORAGE, TOL, pkm_inputs, to_np32
from oracle import oracle as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from deltagrid_b200 import hsru_delta_cuda as ext


def _oracle(d, dtype, want_saved=False):
    r = O.pkm_forward(to_np32(d["v"]), to_np32(d["beta"]), to_np32(d["wk"]), to_np32(d["wq"]),
                      d["idx"].numpy(), to_np32(d["decay"]), to_np32(d["state"]), STORAGE[dtype],
                      want_saved=want_saved)
    return (O.round_to(r[0], STORAGE[dtype]),) + tuple(r[1:])


def _gpu(d, save=False):
    g = {n: t.cuda() for n, t in d.items()}
    return ext.pkm_forward(g["v"], g["beta"], g["wk"], g["wq"], g["idx"], g["decay"], g["state"], save)


@pytest.mark.parametrize("name", ["pkm_g16_k4_f32.npz", "pkm_g32_k8_f32.npz"])
def test_reference_loop_golden(name):
    g = load_golden(name)
    t = {k: torch.from_numpy(g[k]).cuda() for k in ("v", "beta", "wk", "wq", "idx", "decay", "s_init")}
    out, st, _ = ext.pkm_forward(t["v"], t["beta"], t["wk"], t["wq"], t["idx"], t["decay"], t["s_init"])
    assert rel_err(out.cpu().numpy(), g["y"]) < 1e-5
    assert rel_err(st.cpu().numpy(), g["s_final"]) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("G,K,Dh", [(16, 4, 64), (32, 8, 64), (8, 4, 32), (64, 8, 128), (24, 6, 40)])
def test_shapes_and_dtypes(dtype, G, K, Dh):
    d = pkm_inputs(2, 3, 40, G, K, Dh, dtype, dynamic=(G % 16 == 0), seed=G * K + Dh, s_init_scale=0.1)
    out, st, _ = _gpu(d)
    yo, so = _oracle(d, dtype)
    assert rel_err(out.float().cpu().numpy(), yo) < TOL[dtype]
    assert rel_err(st.float().cpu().numpy(), so) < TOL[dtype]


def test_in_place_and_saved_rows():
    d = pkm_inputs(2, 2, 16, 16, 4, 64, torch.float16, seed=2, s_init_scale=0.2)
    g = {n: t.cuda() for n, t in d.items()}
    state = g["state"]
    out, st, saved = ext.pkm_forward(g["v"], g["beta"], g["wk"], g["wq"], g["idx"], g["decay"], state, True)
    assert st.data_ptr() == state.data_ptr()              # updated in place, returned
    yo, so, savedo = _oracle(d, torch.float16, want_saved=True)
    assert saved.shape == (2, 2, 16, 16, 64)
    assert rel_err(saved.float().cpu().numpy(), savedo) < 1e-3      # rows as gathered each step
    assert rel_err(st.float().cpu().numpy(), so) < 1e-3


def test_heavy_row_reuse_ordering():
    # 16 active rows out of 64: most rows recur every few steps, so each step
    # must see the rows its predecessor wrote
    d = pkm_inputs(1, 2, 300, 8, 4, 64, torch.float32, dynamic=True, seed=4)
    out, st, _ = _gpu(d)
    yo, so = _oracle(d, torch.float32)
    assert rel_err(out.cpu().numpy(), yo) < 1e-5
    assert rel_err(st.cpu().numpy(), so) < 1e-5


def test_cfg3_shape_prefix():
    # cfg3 geometry (128 x 128 slots, top-8, Dh 64, fp16 state) on a
    # T prefix and fewer lanes so the CPU oracle stays quick
    d = pkm_inputs(4, 4, 256, 128, 8, 64, torch.float16, seed=7)
    out, st, _ = _gpu(d)
    yo, so = _oracle(d, torch.float16)
    assert rel_err(out.float().cpu().numpy(), yo) < 1e-3
    assert rel_err(st.float().cpu().numpy(), so) < 1e-3


@pytest.mark.parametrize("dynamic", [False, True])
def test_pkm_step(dynamic):
    B, H, G, K, Dh = 3, 2, 16, 4, 32
    d = pkm_inputs(B, H, 1, G, K, Dh, torch.float32, dynamic=dynamic, seed=11, s_init_scale=0.5)
    g = {n: t.cuda() for n, t in d.items()}
    decay = g["decay"][:, :, 0] if dynamic else g["decay"]        # [B,H] as the layer passes it
    y, st = ext.pkm_step(g["v"][:, :, 0], g["beta"][:, :, 0], g["wk"][:, :, 0], g["wq"][:, :, 0],
                         g["idx"][:, :, 0], decay, g["state"])
    yo, so = _oracle(d, torch.float32)
    assert rel_err(y.cpu().numpy(), yo[:, :, 0]) < 1e-5
    assert rel_err(st.cpu().numpy(), so) < 1e-5


def test_reference_step_kernel_case():
    # reference tests/test_sparse_pkm.py:93-133: b,h=2, Dh 32, 16 of 256 slots, decay 0.999
    torch.manual_seed(0)
    b, h, dh, A, total = 2, 2, 32, 16, 256
    v = torch.randn(b, h, dh, device="cuda")
    beta = torch.rand(b, h, device="cuda")
    wk = torch.nn.functional.normalize(torch.randn(b, h, A, device="cuda"), dim=-1)
    wq = torch.randn(b, h, A, device="cuda")
    idx = torch.stack([torch.stack([torch.randperm(total)[:A] for _ in range(h)]) for _ in range(b)]).cuda()
    decay = torch.full((h,), 0.999, device="cuda")
    s0 = torch.randn(b, h, total, dh, device="cuda")
    ex = idx.unsqueeze(-1).expand(b, h, A, dh)
    s_act = torch.gather(s0, 2, ex)
    y_ref = (wq.unsqueeze(-2) @ s_act).squeeze(-2)
    rt = v - (wk.unsqueeze(-2) @ s_act).squeeze(-2)
    s_ref = s0.scatter(2, ex, decay.view(1, h, 1, 1) * s_act + (beta.unsqueeze(-1) * wk).unsqueeze(-1) * rt.unsqueeze(-2))
    y, st = ext.pkm_step(v, beta, wk, wq, idx, decay, s0.clone())
    assert (y - y_ref).abs().max().item() < 1e-5
    assert (st - s_ref).abs().max().item() < 1e-5


def test_out_of_range_index_is_skipped_and_flagged():
    d = pkm_inputs(1, 1, 4, 8, 2, 64, torch.float32, seed=1, s_init_scale=0.3)
    d["idx"][0, 0, 2, 1] = 64          # one past the end: the kernel's bounds check skips it
    ext.device_status("cuda")           # clear
    out, st, _ = _gpu(d)
    assert ext.device_status("cuda") & 0x1
    assert torch.isfinite(out).all() and torch.isfinite(st).all()
