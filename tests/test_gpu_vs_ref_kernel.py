"""Parity against the reference's own CUDA kernels (src/cpp/delta_kernel.cu), built
from the reference sources for sm_100a into oracle/_ref/ by oracle/build_ref_cuda.py.

Same inputs to both extensions; outputs compared with max|a-b|/max|b| at the
north-star tolerances (1e-5 fp32, 1e-3 fp16).  Skipped when the prebuilt
reference extension is absent.
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
TOL = {torch.float32: 1e-5, torch.float16: 1e-3}


def _c(t):
    return t.float().cpu().numpy()


@need_ref
@pytest.mark.parametrize("dtype,B,H,T,S,Dh,dyn", [
    (torch.float32, 4, 4, 512, 64, 64, False),      # cfg1 (the first BASELINE config)
    (torch.float16, 4, 4, 256, 512, 64, False),     # config 1 geometry, fewer lanes
    (torch.float16, 2, 3, 100, 128, 64, True),
    (torch.float32, 2, 2, 64, 256, 32, True),
])
def test_dense_forward_vs_reference_kernel(dtype, B, H, T, S, Dh, dyn):
    d = dense_inputs(B, H, T, S, Dh, dtype, dynamic=dyn, seed=S + T)
    g = {n: (t.cuda() if t is not None else None) for n, t in d.items()}
    args = (g["q"], g["k"], g["v"], g["beta"], g["wk"], g["wq"], g["decay"])
    ro, rs, _, _ = REF.forward(*args, None, False)
    mo, ms, _, _ = ext.forward(*args)
    assert rel_err(_c(mo), _c(ro)) < TOL[dtype]
    assert rel_err(_c(ms), _c(rs)) < TOL[dtype]


@need_ref
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_dense_step_vs_reference_kernel(dtype):
    d = dense_inputs(3, 4, 1, 128, 64, dtype, dynamic=True, seed=2, s_init=True)
    g = {n: t.cuda() for n, t in d.items()}
    args = (g["q"][:, :, 0], g["k"][:, :, 0], g["v"][:, :, 0], g["beta"][:, :, 0], g["wk"][:, :, 0],
            g["wq"][:, :, 0], g["decay"][:, :, 0], g["s_init"])
    ry, rs = REF.step(*args)
    my, ms = ext.step(*args)
    assert rel_err(_c(my), _c(ry)) < TOL[dtype]
    assert rel_err(_c(ms), _c(rs)) < TOL[dtype]


@need_ref
@pytest.mark.parametrize("dtype,G,K,T", [(torch.float16, 128, 8, 256), (torch.float32, 32, 8, 64),
                                         (torch.float16, 16, 4, 200)])
def test_pkm_forward_vs_reference_kernel(dtype, G, K, T):
    d = pkm_inputs(2, 4, T, G, K, 64, dtype, seed=G + T, s_init_scale=0.1)
    g = {n: t.cuda() for n, t in d.items()}
    rs0, ms0 = g["state"].clone(), g["state"].clone()
    ro, rs, _ = REF.pkm_forward(g["v"], g["beta"], g["wk"], g["wq"], g["idx"], g["decay"], rs0, False)
    mo, ms, _ = ext.pkm_forward(g["v"], g["beta"], g["wk"], g["wq"], g["idx"], g["decay"], ms0, False)
    assert rel_err(_c(mo), _c(ro)) < TOL[dtype]
    assert rel_err(_c(ms), _c(rs)) < TOL[dtype]


@need_ref
def test_pkm_step_vs_reference_kernel_static_decay():
    d = pkm_inputs(3, 2, 1, 32, 8, 64, torch.float32, seed=5, s_init_scale=0.4)
    g = {n: t.cuda() for n, t in d.items()}
    a = (g["v"][:, :, 0], g["beta"][:, :, 0], g["wk"][:, :, 0], g["wq"][:, :, 0], g["idx"][:, :, 0], g["decay"])
    ry, rs = REF.pkm_step(*a, g["state"].clone())
    my, ms = ext.pkm_step(*a, g["state"].clone())
    assert rel_err(_c(my), _c(ry)) < 1e-5
    assert rel_err(_c(ms), _c(rs)) < 1e-5


@need_ref
@pytest.mark.parametrize("S,T", [(256, 512), (128, 300), (512, 256)])
def test_dense_bf16_error_not_above_reference_kernel(S, T):
    """bf16 storage: both kernels against the CPU oracle (fp32 state on the bf16 inputs);
    this repository's error may not exceed the reference kernel's, on the fp32 final
    state and the bf16 outputs alike (plus one bf16 ulp of slack on the rounded outputs,
    where either side's rounding of a near-tie can flip)."""
    import numpy as np
    from oracle import oracle as O
    d = dense_inputs(2, 4, T, S, 64, torch.bfloat16, dynamic=True, seed=S + T + 7)
    g = {n: (t.cuda() if t is not None else None) for n, t in d.items()}
    args = (g["q"], g["k"], g["v"], g["beta"], g["wk"], g["wq"], g["decay"])
    ro, rs, _, rsf = REF.forward(*args, None, True)
    mo, ms, _, msf = ext.forward(*args, None, True)
    yo, so = O.dense_forward(*(d[n].float().numpy() for n in ("v", "beta", "wk", "wq", "decay")))
    assert rel_err(_c(msf), so) <= max(rel_err(_c(rsf), so), 1e-3)
    assert rel_err(_c(mo), O.round_to(yo, O.BF16)) <= rel_err(_c(ro), O.round_to(yo, O.BF16)) + 2 ** -8
