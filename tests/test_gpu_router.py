"""Fused PKM router on the GPU against the CPU oracle (same fp32 FMA order: indices
exact) and against the reference layer's router goldens (indices exact outside
documented near-ties, gap < 1e-5)."""
import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err
from oracle import oracle as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from deltagrid_b200 import hsru_delta_cuda as ext
    from deltagrid_b200.route import pkm_route


def _routers(G0, G1, Dh, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(G, Dh, generator=g) / Dh ** 0.5 for G in (G0, G1, G0, G1)]


@pytest.mark.parametrize("G,K,dtype", [(128, 8, torch.float16), (1024, 8, torch.float16),
                                       (64, 4, torch.float32), (32, 8, torch.bfloat16),
                                       # grids of whole 16-row but not 32-row groups, and 32-row blocks
                                       (48, 8, torch.float16), (80, 4, torch.bfloat16), (96, 8, torch.float16),
                                       (160, 8, torch.float16)])
def test_router_vs_oracle(G, K, dtype):
    B, H, T, Dh = 2, 3, 40, 64
    g = torch.Generator().manual_seed(G + K)
    k = torch.nn.functional.normalize(torch.randn(B, H, T, Dh, generator=g), dim=-1).to(dtype)
    q = torch.randn(B, H, T, Dh, generator=g).to(dtype)
    w = _routers(G, G, Dh, 7)
    qs = 0.5 + torch.rand(H, generator=g)
    wk, wq, idx = pkm_route(k.cuda(), q.cuda(), [w[0].cuda(), w[1].cuda()], [w[2].cuda(), w[3].cuda()], K, qs.cuda())
    qsb = qs.view(1, H, 1).expand(B, H, T).numpy()
    wko, wqo, idxo, margin = O.pkm_route(k.float().numpy(), q.float().numpy(), *(x.numpy() for x in w), K,
                                         q_scale=qsb)
    np.testing.assert_array_equal(idx.cpu().numpy(), idxo)          # same fp32 FMA order: exact
    tol = {torch.float32: 1e-5, torch.float16: 1e-3, torch.bfloat16: 8e-3}[dtype]
    assert rel_err(wk.float().cpu().numpy(), wko) < tol
    assert rel_err(wq.float().cpu().numpy(), wqo) < tol


def test_router_vs_reference_layer_golden():
    gld = load_golden("router_g128_k8.npz")
    k = torch.from_numpy(gld["k"]).cuda()
    q = torch.from_numpy(gld["q"]).cuda()
    rk = [torch.from_numpy(gld["router_k0"]).cuda(), torch.from_numpy(gld["router_k1"]).cuda()]
    rq = [torch.from_numpy(gld["router_q0"]).cuda(), torch.from_numpy(gld["router_q1"]).cuda()]
    wk, wq, idx = pkm_route(k, q, rk, rq, 8)
    *_, margin = O.pkm_route(gld["k"], gld["q"], gld["router_k0"], gld["router_k1"], gld["router_q0"],
                             gld["router_q1"], 8)
    # one near-tie in the fixture (margin <= 1e-5); every token's indices are exact
    assert int((margin <= 1e-5).sum()) == 1
    np.testing.assert_array_equal(idx.cpu().numpy(), gld["idx"])
    assert rel_err(wk.cpu().numpy(), gld["wk"]) < 1e-5
    assert rel_err(wq.cpu().numpy(), gld["wq"]) < 1e-5


def test_router_tie_order_lower_index_first():
    # duplicated router rows give exactly equal scores: the lower index must rank first
    Dh, G = 64, 16
    base = torch.randn(G, Dh)
    base[9] = base[2]          # rows 2 and 9 tie, rows 5 and 12 tie
    base[12] = base[5]
    k = torch.randn(1, 1, 8, Dh)
    wk, wq, idx = pkm_route(k.cuda(), k.cuda(), [base.cuda(), base.cuda()], [base.cuda(), base.cuda()], 4)
    _, _, idxo, _ = O.pkm_route(k.numpy(), k.numpy(), base.numpy(), base.numpy(), base.numpy(), base.numpy(), 4)
    np.testing.assert_array_equal(idx.cpu().numpy(), idxo)


def test_routed_forward_matches_two_step_reference():
    B, H, T, Dh, G, K = 2, 2, 64, 64, 32, 8
    g = torch.Generator().manual_seed(3)
    k = torch.nn.functional.normalize(torch.randn(B, H, T, Dh, generator=g), dim=-1).half().cuda()
    q = torch.randn(B, H, T, Dh, generator=g).half().cuda()
    v = torch.nn.functional.normalize(torch.randn(B, H, T, Dh, generator=g), dim=-1).half().cuda()
    beta = torch.sigmoid(torch.randn(B, H, T, generator=g)).half().cuda()
    decay = torch.ones(H, dtype=torch.float16, device="cuda")
    w = [x.cuda() for x in _routers(G, G, Dh, 1)]
    st = torch.zeros(B, H, G * G, Dh, dtype=torch.float16, device="cuda")
    y, st, idx, _ = ext.pkm_fused_forward(k, q, v, beta, w[:2], w[2:], None, decay, st, top_k=K,
                                          grid=(G, G))
    wk, wq, idx2 = pkm_route(k, q, w[:2], w[2:], K)
    st2 = torch.zeros_like(st)
    y2, st2, _ = ext.pkm_forward(v, beta, wk, wq, idx2, decay, st2)
    assert torch.equal(idx, idx2) and torch.equal(y, y2) and torch.equal(st, st2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_tensor_core_router_ties_and_crowded_threshold(dtype):
    # 16-bit keys take the tensor-core router.  Duplicated router rows give exactly equal
    # scores (lower index first); a block of 40 identical rows puts far more than 16
    # candidates inside the error window, so those tokens take the exact full rescan.
    Dh, G, K = 64, 256, 8
    g = torch.Generator().manual_seed(11)
    w = torch.randn(G, Dh, generator=g) / Dh ** 0.5
    w[9] = w[2]
    w[130] = w[77]
    w[200:240] = w[199]
    k = torch.nn.functional.normalize(torch.randn(1, 2, 96, Dh, generator=g), dim=-1)
    k[0, 1, :40] = torch.nn.functional.normalize(w[199], dim=0)          # these tokens prefer rows 199..239
    k = k.to(dtype)
    q = torch.randn(1, 2, 96, Dh, generator=g).to(dtype)
    wk, wq, idx = pkm_route(k.cuda(), q.cuda(), [w.cuda(), w.cuda()], [w.cuda(), w.cuda()], K)
    _, _, idxo, _ = O.pkm_route(k.float().numpy(), q.float().numpy(), w.numpy(), w.numpy(), w.numpy(), w.numpy(), K)
    np.testing.assert_array_equal(idx.cpu().numpy(), idxo)


def test_router_wait_timeout_marks_tokens():
    """With the wait budget at zero the tensor-core router's first wait gives up: it
    drains the copies and MMAs it issued, writes index -1 (out of range) and zero
    weights for every token, and returns; the next call with the normal budget is
    exact again."""
    B, H, T, Dh, G, K = 2, 2, 200, 64, 128, 8
    g = torch.Generator().manual_seed(21)
    k = torch.nn.functional.normalize(torch.randn(B, H, T, Dh, generator=g), dim=-1).half().cuda()
    q = torch.randn(B, H, T, Dh, generator=g).half().cuda()
    w = [x.cuda() for x in _routers(G, G, Dh, 5)]
    old = ext.set_wait_limit(0)
    try:
        wk, wq, idx = pkm_route(k, q, w[:2], w[2:], K)
        torch.cuda.synchronize()
    finally:
        ext.set_wait_limit(old)
    assert bool((idx == -1).all()) and float(wk.abs().max()) == 0.0 and float(wq.abs().max()) == 0.0
    wk, wq, idx = pkm_route(k, q, w[:2], w[2:], K)
    wko, wqo, idxo, _ = O.pkm_route(k.float().cpu().numpy(), q.float().cpu().numpy(),
                                    *[x.cpu().numpy() for x in w], K)
    np.testing.assert_array_equal(idx.cpu().numpy(), idxo)
