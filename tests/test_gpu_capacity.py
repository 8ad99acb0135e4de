"""Associative recall at scale through the whole GPU path: routing (dg_pkm_route),
the hazard pre-pass and the PKM recurrence.

cfg4's stream (the fourth BASELINE config): per lane, 100,000 writes of random unit-norm key /
value pairs (beta = 1, alpha = 1) into a 1024 x 1024 grid (1,048,576 slots, top-8
per axis, 64 active slots), then 10,000 reads of uniformly chosen earlier keys
(beta = 0, the query routed like its key); a read succeeds when cos(y, v) > 0.8.
The reference reports for this regime (README.md:181, 100k facts on 1M slots)
a mean cosine of 0.8930 and 90.5 % recall, and on the 128 x 128 grid with top-4
(16 active slots) 0.9334 and 98.2 % after 2,000 facts.  This is a quality check
of the path, not a parity test: keys here are routed directly (no projections),
so the bounds sit a little below what this path measures.
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from deltagrid_b200 import hsru_delta_cuda as ext
    from deltagrid_b200.route import pkm_route


def capacity_run(G, K, n_write, n_read, lanes=2, chunk=16384, seed=0):
    """(mean cosine, recall at cos > 0.8) of n_read reads after n_write writes, per lane."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    Dh, H = 64, lanes
    routers = [torch.randn(G, Dh, device=dev, generator=g) / Dh ** 0.5 for _ in range(2)]
    keys = F.normalize(torch.randn(1, H, n_write, Dh, device=dev, generator=g), dim=-1).half()
    vals = F.normalize(torch.randn(1, H, n_write, Dh, device=dev, generator=g), dim=-1).half()
    state = torch.zeros(1, H, G * G, Dh, device=dev, dtype=torch.float16)
    decay = torch.ones(H, device=dev, dtype=torch.float16)
    for t0 in range(0, n_write, chunk):
        k = keys[:, :, t0:t0 + chunk].contiguous()
        T = k.shape[2]
        wk, wq, idx = pkm_route(k, k, routers, routers, K)
        beta = torch.ones(1, H, T, device=dev, dtype=torch.float16)
        ext.pkm_forward(vals[:, :, t0:t0 + T].contiguous(), beta, wk, wq, idx, decay, state)
    pick = torch.randint(0, n_write, (H, n_read), device=dev, generator=g)
    q = torch.stack([keys[0, h, pick[h]] for h in range(H)]).unsqueeze(0).contiguous()
    want = torch.stack([vals[0, h, pick[h]] for h in range(H)]).float()
    wk, wq, idx = pkm_route(q, q, routers, routers, K)
    zeros = torch.zeros(1, H, n_read, device=dev, dtype=torch.float16)
    y, _, _ = ext.pkm_forward(torch.zeros_like(q), zeros, wk, wq, idx, decay, state)
    torch.cuda.synchronize()
    assert ext.device_status(clear=True) == 0
    cos = F.cosine_similarity(y[0].float(), want, dim=-1)
    return float(cos.mean()), float((cos > 0.8).float().mean())


def test_recall_1m_slots_100k_facts():
    mean_cos, recall = capacity_run(1024, 8, 100_000, 10_000)       # measured on B200: 0.894, 91.6 %
    assert mean_cos > 0.87 and recall > 0.86, (mean_cos, recall)


def test_recall_16k_slots_2k_facts():
    mean_cos, recall = capacity_run(128, 4, 2_000, 2_000)           # measured on B200: 0.924, 96.3 %
    assert mean_cos > 0.90 and recall > 0.93, (mean_cos, recall)
