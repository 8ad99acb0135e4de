"""Seeded synthetic inputs with the shapes and distributions of the BASELINE configs.

Dense: q, k, v ~ N(0,1), k L2-normalised, beta = sigmoid(N(0,1)); with
slots != Dh the slot routing of memory.py:233-236 (wk = normalize(k P^T),
wq = q P^T, P an orthogonal slots x Dh matrix).  PKM: values unit-norm,
Kronecker keys from two top-k axes, indices i0 * G1 + i1 (distinct per step).
Everything is generated on the CPU from torch.Generator seeds.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def orthogonal(rows: int, cols: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    w = torch.empty(rows, cols)
    torch.nn.init.orthogonal_(w, generator=g)
    return w


def dense_inputs(B, H, T, S, Dh, dtype=torch.float32, dynamic=False, seed=0, s_init=False,
                 static_decay=1.0):
    g = torch.Generator().manual_seed(seed)
    k = F.normalize(torch.randn(B, H, T, Dh, generator=g), dim=-1)
    q = torch.randn(B, H, T, Dh, generator=g)
    v = torch.randn(B, H, T, Dh, generator=g)
    beta = torch.sigmoid(torch.randn(B, H, T, generator=g))
    if S == Dh:
        wk, wq = k, q
    else:
        P = orthogonal(S, Dh, seed + 1)
        wk = F.normalize(k @ P.T, dim=-1)
        wq = q @ P.T
    if dynamic:
        decay = 0.99 + 0.01 * torch.sigmoid(torch.randn(B, H, T, generator=g))
    else:
        decay = torch.full((H,), float(static_decay))
    s0 = 0.1 * torch.randn(B, H, S, Dh, generator=g) if s_init else None
    d = dict(q=q, k=k, v=v, beta=beta, wk=wk, wq=wq, decay=decay, s_init=s0)
    return {n: (t.to(dtype) if t is not None else None) for n, t in d.items()}


def pkm_inputs(B, H, T, G, K, Dh, dtype=torch.float16, dynamic=False, seed=0, s_init_scale=0.0):
    g = torch.Generator().manual_seed(seed)
    i0 = torch.rand(B, H, T, G, generator=g).argsort(-1)[..., :K]
    i1 = torch.rand(B, H, T, G, generator=g).argsort(-1)[..., :K]
    idx = (i0.unsqueeze(-1) * G + i1.unsqueeze(-2)).flatten(-2).to(torch.int64)
    u0 = F.normalize(torch.rand(B, H, T, K, generator=g) + 0.1, dim=-1)
    u1 = F.normalize(torch.rand(B, H, T, K, generator=g) + 0.1, dim=-1)
    wk = (u0.unsqueeze(-1) * u1.unsqueeze(-2)).flatten(-2)
    wq = torch.randn(B, H, T, K * K, generator=g) / K
    v = F.normalize(torch.randn(B, H, T, Dh, generator=g), dim=-1)
    beta = torch.sigmoid(torch.randn(B, H, T, generator=g))
    decay = (0.99 + 0.01 * torch.sigmoid(torch.randn(B, H, T, generator=g))) if dynamic else torch.ones(H)
    state = s_init_scale * torch.randn(B, H, G * G, Dh, generator=g)
    d = dict(v=v, beta=beta, wk=wk, wq=wq, decay=decay, state=state)
    out = {n: t.to(dtype) for n, t in d.items()}
    out["idx"] = idx
    return out


def to_np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


STORAGE = {torch.float32: 0, torch.float64: 1, torch.float16: 2, torch.bfloat16: 3}

# parity tolerance per storage dtype: max|a-b| / max|b|
TOL = {torch.float32: 1e-5, torch.float64: 1e-5, torch.float16: 1e-3, torch.bfloat16: 8e-3}
