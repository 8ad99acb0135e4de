"""Slot routing kernel (dg_dense_route, csrc/slot_route.cu) against a plain PyTorch
fp32 evaluation of DeltaGridLayer._route_dense's slot-projection branch and the
q_scale multiply (src/modules/memory.py:233-236, :490-492): wk = normalize(k P_k^T),
wq = (q P_q^T) q_scale[h].  Bar, max|a-b|/max|b| per output: 1e-3 for fp16 (one
output rounding, 2^-11 relative, on fp32 products) and 8e-3 for bf16 (2^-8)."""
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_err

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from deltagrid_b200 import hsru_delta_cuda as ext
    from deltagrid_b200.route import dense_route

TOL = {torch.float16: 1e-3, torch.bfloat16: 8e-3}


def _ref(k, q, pk, pq, qs):
    wk = F.normalize(k.float() @ pk.float().T, p=2, dim=-1)
    wq = q.float() @ pq.float().T
    if qs is not None:
        wq = wq * qs.float().view(1, -1, 1, 1)
    return wk, wq


def _inputs(B, H, T, S, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    k = F.normalize(torch.randn(B, H, T, 64, generator=g), dim=-1).to(dtype).cuda()
    q = torch.randn(B, H, T, 64, generator=g).to(dtype).cuda()
    pk = torch.empty(S, 64)
    torch.nn.init.orthogonal_(pk, generator=g)
    pq = (torch.randn(S, 64, generator=g) / 8)
    qs = (0.5 + torch.rand(H, generator=g)).cuda()
    return k, q, pk.to(dtype).cuda(), pq.to(dtype).cuda(), qs


@pytest.mark.parametrize("S", [64, 128, 192, 256, 384, 512])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_dense_route_against_torch(S, dtype):
    k, q, pk, pq, qs = _inputs(2, 3, 100, S, dtype, seed=S)        # 600 tokens: a ragged last tile
    wk, wq = dense_route(k, q, pk, pq, qs)
    torch.cuda.synchronize()
    rk, rq = _ref(k, q, pk, pq, qs)
    assert wk.dtype == dtype and wk.shape == (2, 3, 100, S)
    assert rel_err(wk.float().cpu(), rk.cpu()) < TOL[dtype]
    assert rel_err(wq.float().cpu(), rq.cpu()) < TOL[dtype]
    assert ext.device_status() == 0


def test_dense_route_many_tiles_no_q_scale():
    """More tiles than SMs (each CTA takes several in turn), q_scale absent."""
    k, q, pk, pq, _ = _inputs(4, 16, 4096, 512, torch.float16, seed=1)
    wk, wq = dense_route(k, q, pk, pq, None)
    torch.cuda.synchronize()
    rk, rq = _ref(k, q, pk, pq, None)
    assert rel_err(wk.float().cpu(), rk.cpu()) < 1e-3
    assert rel_err(wq.float().cpu(), rq.cpu()) < 1e-3


def test_dense_fused_forward_uses_kernel_and_matches_torch_route():
    """dense_fused_forward (kernel routing) against forward on torch-routed wk / wq."""
    B, H, T, S = 2, 4, 256, 512
    k, q, pk, pq, qs = _inputs(B, H, T, S, torch.float16, seed=3)
    g = torch.Generator().manual_seed(4)
    v = torch.randn(B, H, T, 64, generator=g).half().cuda()
    beta = torch.sigmoid(torch.randn(B, H, T, generator=g)).half().cuda()
    decay = torch.ones(H, dtype=torch.float16, device="cuda")
    out, s, _, _ = ext.dense_fused_forward(k, q, v, beta, pk, pq, qs, decay)
    rk, rq = _ref(k, q, pk, pq, qs)
    out2, s2, _, _ = ext.forward(q, k, v, beta, rk.half(), rq.half(), decay)
    torch.cuda.synchronize()
    assert rel_err(out.float().cpu(), out2.float().cpu()) < 2e-3
    assert rel_err(s.float().cpu(), s2.float().cpu()) < 2e-3


def test_dense_route_wait_timeout_flags_status():
    """Wait budget zero: the kernel's first wait gives up, it drains what it issued,
    flags DG_DEVCHK_TIMEOUT and returns; the next call is exact again."""
    k, q, pk, pq, qs = _inputs(1, 2, 300, 256, torch.float16, seed=5)
    ext.device_status()
    old = ext.set_wait_limit(0)
    try:
        dense_route(k, q, pk, pq, qs)
        torch.cuda.synchronize()
    finally:
        ext.set_wait_limit(old)
    assert ext.device_status() & 0x4
    wk, wq = dense_route(k, q, pk, pq, qs)
    torch.cuda.synchronize()
    assert ext.device_status() == 0
    rk, rq = _ref(k, q, pk, pq, qs)
    assert rel_err(wk.float().cpu(), rk.cpu()) < 1e-3


def test_dense_route_rejects_uncovered_shapes():
    k, q, pk, pq, qs = _inputs(1, 1, 16, 96, torch.float16, seed=6)
    with pytest.raises(RuntimeError):
        dense_route(k, q, pk, pq, qs)
