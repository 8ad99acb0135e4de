"""Q16.16 fixed-point recurrence on the GPU, bit-exact with the reference engine.

Torch int32 CUDA tensors in the lanes-first layout of the engine's recurrence
core (one lane = one (context, head)); see dg_fxp_dense_forward /
dg_fxp_pkm_forward in include/deltagrid_b200.h.  The state is updated in place.
"""
from __future__ import annotations

import torch

from . import _lib


def _chk(*ts):
    for t in ts:
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.int32 or not t.is_contiguous():
            raise RuntimeError("fxp tensors must be contiguous int32 CUDA tensors")


def dense_forward(wk, wq, v, beta, alpha, state):
    """wk, wq [L,T,S]; v [L,T,Dh]; beta, alpha [L,T]; state [L,S,Dh] (in place). Returns (y, state)."""
    _chk(wk, wq, v, beta, alpha, state)
    L, T, S = wk.shape
    Dh = v.shape[-1]
    y = torch.empty((L, T, Dh), dtype=torch.int32, device=v.device)
    with torch.cuda.device(v.device):
        _lib.call("dg_fxp_dense_forward", L, T, S, Dh, wk.data_ptr(), wq.data_ptr(), v.data_ptr(),
                  beta.data_ptr(), alpha.data_ptr(), state.data_ptr(), y.data_ptr(),
                  torch.cuda.current_stream(v.device).cuda_stream)
    return y, state


def pkm_forward(wk, wq, idx, v, beta, alpha, state, status=None):
    """wk, wq, idx [L,T,A] (int32 slots); v [L,T,Dh]; beta, alpha [L,T]; state [L,total,Dh] in place."""
    _chk(wk, wq, idx, v, beta, alpha, state)
    L, T, A = wk.shape
    Dh = v.shape[-1]
    total = state.shape[1]
    y = torch.empty((L, T, Dh), dtype=torch.int32, device=v.device)
    with torch.cuda.device(v.device):
        _lib.call("dg_fxp_pkm_forward", L, T, A, total, Dh, wk.data_ptr(), wq.data_ptr(), idx.data_ptr(),
                  v.data_ptr(), beta.data_ptr(), alpha.data_ptr(), state.data_ptr(), y.data_ptr(),
                  status.data_ptr() if status is not None else None,
                  torch.cuda.current_stream(v.device).cuda_stream)
    return y, state
