"""Analytic backward passes, dense (dg_dense_backward) and Sparse Delta-PKM
(dg_pkm_backward), reached through hsru_delta_cuda.backward / .pkm_backward.

Two independent checks of every gradient:
- the reference's own CUDA backward kernels (src/cpp/delta_kernel.cu:364-558 and
  :971-1072, built from the reference sources into oracle/_ref/), fed the same saved
  tensors; bar max|a-b|/max|b| <= 1e-5 in fp32, 1e-3 in fp16 (4e-3 for the
  reference's fp16 atomic sums of a static decay gradient);
- torch autograd through a plain PyTorch fp64 loop of the same recurrence
  (memory.py:524-539), on the storage-quantised inputs; bar 1e-4 in fp32 (the
  backward reconstructs S_{t-1} from S_t step by step in fp32, as the reference does)
  and 2e-3 in fp16.
The PKM reference kernel never writes the gradient of a static [H] decay, so that
output is only checked against autograd.
"""
import pytest
import torch

from conftest import rel_err
from inputs import dense_inputs, pkm_inputs
from oracle.build_ref_cuda import load_prebuilt

pytestmark = pytest.mark.gpu

REF = load_prebuilt() if torch.cuda.is_available() else None
if torch.cuda.is_available():
    from deltagrid_b200 import hsru_delta_cuda as ext

need_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref/ref_hsru_delta_cuda.so not built")
TOL_REF = {torch.float32: 1e-5, torch.float16: 1e-3}
TOL_AG = {torch.float32: 1e-4, torch.float16: 2e-3, torch.bfloat16: 1.6e-2}


def _np(t):
    return t.detach().double().cpu().numpy()


def _dense_case(dtype, B, H, T, S, Dh, dyn, seed, with_gsf=True, s_init=True, static_decay=1.0):
    d = dense_inputs(B, H, T, S, Dh, dtype, dynamic=dyn, seed=seed, s_init=s_init, static_decay=static_decay)
    g = {n: (t.cuda() if t is not None else None) for n, t in d.items()}
    gen = torch.Generator().manual_seed(seed + 99)
    gy = torch.randn(B, H, T, Dh, generator=gen).to(dtype).cuda()
    gsf = (0.1 * torch.randn(B, H, S, Dh, generator=gen)).to(dtype).cuda() if with_gsf else None
    out, s_fin, err, sff = ext.forward(g["q"], g["k"], g["v"], g["beta"], g["wk"], g["wq"], g["decay"],
                                       g["s_init"], True)
    sff = sff if sff is not None else s_fin.float()
    return g, gy, gsf, sff, err


def _dense_autograd(g, gy, gsf):
    """fp64 loop of y_t = wq_t.S, r_t = v_t - wk_t.S, S <- alpha S + beta wk r^T, with autograd."""
    v, beta, wk, wq, decay = (g[n].double().detach().requires_grad_(True) for n in ("v", "beta", "wk", "wq", "decay"))
    s0 = g["s_init"].double().detach().requires_grad_(True) if g["s_init"] is not None else None
    B, H, T, Dh = v.shape
    S = wk.shape[-1]
    st = s0 if s0 is not None else torch.zeros(B, H, S, Dh, dtype=torch.float64, device=v.device)
    ys = []
    for t in range(T):
        a = decay[:, :, t] if decay.dim() == 3 else decay.view(1, H).expand(B, H)
        ys.append(torch.einsum("bhs,bhsd->bhd", wq[:, :, t], st))
        r = v[:, :, t] - torch.einsum("bhs,bhsd->bhd", wk[:, :, t], st)
        st = a[..., None, None] * st + beta[:, :, t, None, None] * wk[:, :, t, :, None] * r[:, :, None, :]
    loss = (torch.stack(ys, 2) * gy.double()).sum()
    if gsf is not None:
        loss = loss + (st * gsf.double()).sum()
    loss.backward()
    return dict(v=v.grad, beta=beta.grad, wk=wk.grad, wq=wq.grad, decay=decay.grad,
                s_init=s0.grad if s0 is not None else None)


DENSE_CASES = [
    # dtype, B, H, T, S, Dh, dynamic, static decay
    (torch.float32, 2, 2, 64, 64, 64, False, 1.0),
    (torch.float32, 2, 3, 100, 384, 32, False, 0.999),
    (torch.float32, 1, 2, 48, 512, 64, True, 1.0),      # state and adjoint in the fp32 workspace
    (torch.float16, 2, 2, 64, 512, 64, True, 1.0),
    (torch.float16, 2, 2, 80, 128, 64, False, 1.0),
]


@pytest.mark.parametrize("dtype,B,H,T,S,Dh,dyn,sd", DENSE_CASES)
def test_dense_backward_vs_autograd(dtype, B, H, T, S, Dh, dyn, sd):
    g, gy, gsf, sff, err = _dense_case(dtype, B, H, T, S, Dh, dyn, seed=T + S, static_decay=sd)
    gv, gb, gwk, gwq, gd, gsi = ext.backward(gy, gsf, g["v"], g["beta"], g["wk"], g["wq"], g["decay"], sff, err, True)
    ag = _dense_autograd(g, gy, gsf)
    tol = TOL_AG[dtype]
    for name, ours in (("v", gv), ("beta", gb), ("wk", gwk), ("wq", gwq), ("decay", gd), ("s_init", gsi)):
        assert rel_err(_np(ours), _np(ag[name])) < tol, name


@need_ref
@pytest.mark.parametrize("dtype,B,H,T,S,Dh,dyn,sd", DENSE_CASES)
def test_dense_backward_vs_reference_kernel(dtype, B, H, T, S, Dh, dyn, sd):
    g, gy, gsf, sff, err = _dense_case(dtype, B, H, T, S, Dh, dyn, seed=T + S + 1, static_decay=sd)
    args = (gy, gsf, g["v"], g["beta"], g["wk"], g["wq"], g["decay"], sff, err, True)
    ours = ext.backward(*args)
    ref = REF.backward(*args)
    torch.cuda.synchronize()
    for i, name in enumerate(("v", "beta", "wk", "wq", "decay", "s_init")):
        tol = TOL_REF[dtype] * (4 if (name == "decay" and dtype == torch.float16 and not dyn) else 1)
        assert rel_err(_np(ours[i]), _np(ref[i])) < tol, name


def test_dense_backward_without_state_gradients():
    g, gy, _, sff, err = _dense_case(torch.float32, 1, 2, 32, 64, 64, False, seed=5, with_gsf=False, s_init=False)
    gv, gb, gwk, gwq, gd, gsi = ext.backward(gy, None, g["v"], g["beta"], g["wk"], g["wq"], g["decay"], sff, err)
    assert gsi is None
    ag = _dense_autograd(g, gy, None)
    for name, ours in (("v", gv), ("beta", gb), ("wk", gwk), ("wq", gwq), ("decay", gd)):
        assert rel_err(_np(ours), _np(ag[name])) < TOL_AG[torch.float32], name


def _pkm_case(dtype, B, H, T, G, K, Dh, dyn, seed):
    d = pkm_inputs(B, H, T, G, K, Dh, dtype, dynamic=dyn, seed=seed, s_init_scale=0.05)
    g = {n: t.cuda() for n, t in d.items()}
    state0 = g["state"].clone()
    out, st, saved = ext.pkm_forward(g["v"], g["beta"], g["wk"], g["wq"], g["idx"], g["decay"], g["state"], True)
    gen = torch.Generator().manual_seed(seed + 7)
    gy = torch.randn(B, H, T, Dh, generator=gen).to(dtype).cuda()
    gfin = (0.1 * torch.randn(B, H, G * G, Dh, generator=gen)).to(dtype).cuda()
    return g, state0, saved, gy, gfin


def _pkm_autograd(g, state0, gy, gfin):
    """fp64 loop: rows = S[idx]; y = wq.rows; r = v - wk.rows; S[idx] = alpha rows + beta wk r^T."""
    v, beta, wk, wq, decay = (g[n].double().detach().requires_grad_(True) for n in ("v", "beta", "wk", "wq", "decay"))
    s0 = state0.double().detach().requires_grad_(True)
    B, H, T, Dh = v.shape
    idx = g["idx"]
    st = s0
    ys = []
    for t in range(T):
        a = decay[:, :, t] if decay.dim() == 3 else decay.view(1, H).expand(B, H)
        it = idx[:, :, t, :, None].expand(-1, -1, -1, Dh)
        rows = torch.gather(st, 2, it)
        ys.append(torch.einsum("bha,bhad->bhd", wq[:, :, t], rows))
        r = v[:, :, t] - torch.einsum("bha,bhad->bhd", wk[:, :, t], rows)
        new = a[..., None, None] * rows + beta[:, :, t, None, None] * wk[:, :, t, :, None] * r[:, :, None, :]
        st = st.scatter(2, it, new)
    loss = (torch.stack(ys, 2) * gy.double()).sum() + (st * gfin.double()).sum()
    loss.backward()
    return dict(v=v.grad, beta=beta.grad, wk=wk.grad, wq=wq.grad, decay=decay.grad, state=s0.grad)


PKM_CASES = [
    # dtype, B, H, T, G, K, Dh, dynamic
    (torch.float32, 2, 2, 48, 16, 4, 64, True),
    (torch.float32, 1, 3, 40, 8, 4, 32, False),     # 64 slots: rows revisited every few steps
    (torch.float32, 2, 1, 32, 32, 8, 64, True),     # 64 active rows per step
    (torch.float32, 1, 2, 24, 16, 4, 128, False),
]


@pytest.mark.parametrize("dtype,B,H,T,G,K,Dh,dyn", PKM_CASES)
def test_pkm_backward_vs_autograd(dtype, B, H, T, G, K, Dh, dyn):
    g, state0, saved, gy, gfin = _pkm_case(dtype, B, H, T, G, K, Dh, dyn, seed=T + G)
    gv, gb, gwk, gwq, gd, gs = ext.pkm_backward(gy, g["v"], g["beta"], g["wk"], g["wq"], g["idx"], g["decay"],
                                                saved, G * G, gfin, True)
    ag = _pkm_autograd(g, state0, gy, gfin)
    for name, ours in (("v", gv), ("beta", gb), ("wk", gwk), ("wq", gwq), ("decay", gd), ("state", gs)):
        assert rel_err(_np(ours), _np(ag[name])) < TOL_AG[dtype], name


@need_ref
@pytest.mark.parametrize("dtype,dyn", [(torch.float32, True), (torch.float16, True), (torch.float16, False),
                                       (torch.float32, False)])
def test_pkm_backward_vs_reference_kernel(dtype, dyn):
    B, H, T, G, K, Dh = 2, 2, 64, 16, 8, 64
    g, state0, saved, gy, gfin = _pkm_case(dtype, B, H, T, G, K, Dh, dyn, seed=11 + int(dyn))
    args = (gy, g["v"], g["beta"], g["wk"], g["wq"], g["idx"], g["decay"], saved, G * G, gfin, True)
    ours = ext.pkm_backward(*args)
    ref = REF.pkm_backward(*args)
    torch.cuda.synchronize()
    names = ("v", "beta", "wk", "wq", "decay", "state")
    for i, name in enumerate(names):
        if name == "decay" and not dyn:
            continue                                   # the reference leaves a static decay gradient unwritten
        assert rel_err(_np(ours[i]), _np(ref[i])) < TOL_REF[dtype], name


def test_pkm_backward_defaults_and_no_decay_gradient():
    B, H, T, G, K, Dh = 1, 2, 16, 8, 4, 64
    g, state0, saved, gy, _ = _pkm_case(torch.float32, B, H, T, G, K, Dh, False, seed=3)
    gv, gb, gwk, gwq, gd, gs = ext.pkm_backward(gy, g["v"], g["beta"], g["wk"], g["wq"], g["idx"], g["decay"],
                                                saved, G * G)
    assert gd is None and gs.shape == (B, H, G * G, Dh)
    ag = _pkm_autograd(g, state0, gy, torch.zeros_like(gs))
    for name, ours in (("v", gv), ("beta", gb), ("wk", gwk), ("wq", gwq), ("state", gs)):
        assert rel_err(_np(ours), _np(ag[name])) < TOL_AG[torch.float32], name


def test_backward_rejects_host_tensors():
    g, gy, gsf, sff, err = _dense_case(torch.float32, 1, 1, 8, 64, 64, False, seed=1)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        ext.backward(gy.cpu(), gsf, g["v"], g["beta"], g["wk"], g["wq"], g["decay"], sff, err)
