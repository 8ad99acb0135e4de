"""dense_fused_forward: the dense layer's slot routing (memory.py:233-236 and the
q_scale multiply of :490-492) followed by the recurrence, from k and q.

Checked: the result is exactly forward() on the wk / wq that the slot-routing kernel
forms (route.dense_route); those are within one storage rounding of torch's
F.linear / F.normalize routing; and the result matches the CPU oracle run on the
routed (storage-rounded) wk / wq within the fp16 bar of 1e-3, at cfg2's geometry
(512 slots, Dh 64) on a few lanes.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_err
from inputs import orthogonal, to_np32
from oracle import oracle as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from deltagrid_b200 import hsru_delta_cuda as ext


def _inputs(B, H, T, S, Dh, seed):
    g = torch.Generator().manual_seed(seed)
    k = F.normalize(torch.randn(B, H, T, Dh, generator=g), dim=-1).half().cuda()
    q = torch.randn(B, H, T, Dh, generator=g).half().cuda()
    v = torch.randn(B, H, T, Dh, generator=g).half().cuda()
    beta = torch.sigmoid(torch.randn(B, H, T, generator=g)).half().cuda()
    pk = orthogonal(S, Dh, seed + 1).half().cuda()
    pq = orthogonal(S, Dh, seed + 2).half().cuda()
    qs = (1.0 + 0.1 * torch.randn(H, generator=g)).half().cuda()
    decay = (0.99 + 0.01 * torch.sigmoid(torch.randn(B, H, T, generator=g))).half().cuda()
    return k, q, v, beta, pk, pq, qs, decay


@pytest.mark.parametrize("S,T", [(512, 512), (256, 200)])
def test_dense_fused_equals_forward_on_routed_keys(S, T):
    k, q, v, beta, pk, pq, qs, decay = _inputs(2, 3, T, S, 64, seed=S + T)
    from deltagrid_b200.route import dense_route
    o1, s1, _, _ = ext.dense_fused_forward(k, q, v, beta, pk, pq, qs, decay)
    wk, wq = dense_route(k, q, pk, pq, qs)
    o2, s2, _, _ = ext.forward(q, k, v, beta, wk, wq, decay)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    tk = F.normalize(F.linear(k, pk), p=2, dim=-1)
    tq = F.linear(q, pq) * qs.view(1, -1, 1, 1)
    assert rel_err(wk.float().cpu().numpy(), tk.float().cpu().numpy()) < 1e-3
    assert rel_err(wq.float().cpu().numpy(), tq.float().cpu().numpy()) < 1e-3
    yo, so = O.dense_forward(to_np32(v), to_np32(beta), to_np32(wk), to_np32(wq), to_np32(decay))
    assert rel_err(o1.float().cpu().numpy(), O.round_to(yo, O.F16)) < 1e-3
    assert rel_err(s1.float().cpu().numpy(), O.round_to(so, O.F16)) < 1e-3


def test_dense_fused_without_slot_projection():
    k, q, v, beta, _, _, _, decay = _inputs(1, 2, 128, 64, 64, seed=4)
    o1, s1, _, _ = ext.dense_fused_forward(k, q, v, beta, None, None, None, decay)
    o2, s2, _, _ = ext.forward(q, k, v, beta, k, q, decay)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    with pytest.raises(RuntimeError):
        ext.dense_fused_forward(k, q, v, beta, torch.zeros(64, 64, device="cuda"), None, None, decay)
