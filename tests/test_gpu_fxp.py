"""Q16.16 recurrence on the GPU: bit-exact against the reference engine's exports
(golden engine_fxp_*.npz) and against the oracle on larger random cases."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import oracle as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from deltagrid_b200 import fxp


def _lanes(e, name, T, H, last):
    return np.ascontiguousarray(e[name].reshape(T, H, last).transpose(1, 0, 2))


def _cu(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).cuda()


@pytest.mark.parametrize("name", ["engine_fxp_dense_dyn.npz", "engine_fxp_slotproj.npz", "engine_fxp_pkm.npz"])
def test_engine_golden_bit_exact(name):
    e = load_golden(name)
    mode, H, Dh = int(e["mode"]), int(e["H"]), int(e["Dh"])
    T, A = e["wk"].shape[0], e["wk"].shape[-1]
    wk, wq, v = _lanes(e, "wk", T, H, A), _lanes(e, "wq", T, H, A), _lanes(e, "v", T, H, Dh)
    beta, alpha = e["beta"].T, e["alpha"].T
    state = torch.zeros(e["state"].shape, dtype=torch.int32, device="cuda")
    if mode == 2:
        y, st = fxp.pkm_forward(_cu(wk), _cu(wq), _cu(_lanes(e, "idx", T, H, A)), _cu(v), _cu(beta), _cu(alpha), state)
    else:
        y, st = fxp.dense_forward(_cu(wk), _cu(wq), _cu(v), _cu(beta), _cu(alpha), state)
    np.testing.assert_array_equal(y.cpu().numpy(), _lanes(e, "y", T, H, Dh))
    np.testing.assert_array_equal(st.cpu().numpy(), e["state"])


def _rand_q(rs, shape, scale):
    return (rs.randn(*shape) * scale * 65536).astype(np.int32)


@pytest.mark.parametrize("S,Dh", [(64, 64), (256, 64), (512, 64), (100, 40)])
def test_dense_random_bit_exact(S, Dh):
    rs = np.random.RandomState(S + Dh)
    L, T = 6, 50
    wk = _rand_q(rs, (L, T, S), 1 / np.sqrt(S))
    wq = _rand_q(rs, (L, T, S), 1 / np.sqrt(S))
    v = _rand_q(rs, (L, T, Dh), 1.0)
    beta = (rs.rand(L, T) * 65536).astype(np.int32)
    alpha = (65536 - rs.randint(0, 600, (L, T))).astype(np.int32)
    s0 = _rand_q(rs, (L, S, Dh), 0.1)
    yo, so = O.fxp_dense_forward(wk, wq, v, beta, alpha, s0)
    y, st = fxp.dense_forward(_cu(wk), _cu(wq), _cu(v), _cu(beta), _cu(alpha), _cu(s0))
    np.testing.assert_array_equal(y.cpu().numpy(), yo)
    np.testing.assert_array_equal(st.cpu().numpy(), so)


@pytest.mark.parametrize("G,K,Dh", [(16, 4, 64), (32, 8, 64), (8, 4, 32)])
def test_pkm_random_bit_exact(G, K, Dh):
    rs = np.random.RandomState(G * K)
    L, T, A = 4, 120, K * K
    idx = np.empty((L, T, A), np.int32)
    for l in range(L):
        for t in range(T):
            a0 = rs.choice(G, K, replace=False)
            a1 = rs.choice(G, K, replace=False)
            idx[l, t] = (a0[:, None] * G + a1[None, :]).ravel()
    wk = (np.abs(rs.randn(L, T, A)) / K * 65536).astype(np.int32)
    wq = _rand_q(rs, (L, T, A), 1 / K)
    v = _rand_q(rs, (L, T, Dh), 1.0)
    beta = (rs.rand(L, T) * 65536).astype(np.int32)
    alpha = (65536 - rs.randint(0, 600, (L, T))).astype(np.int32)
    s0 = _rand_q(rs, (L, G * G, Dh), 0.1)
    yo, so = O.fxp_pkm_forward(wk, wq, idx, v, beta, alpha, s0)
    y, st = fxp.pkm_forward(_cu(wk), _cu(wq), _cu(idx), _cu(v), _cu(beta), _cu(alpha), _cu(s0))
    np.testing.assert_array_equal(y.cpu().numpy(), yo)
    np.testing.assert_array_equal(st.cpu().numpy(), so)
