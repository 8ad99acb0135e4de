"""Fused routing kernels in front of the recurrences.

`pkm_route` is the GPU counterpart of DeltaGridLayer._route_sparse_pkm
(src/modules/memory.py:240-289, two axes) including the q_scale multiply of
memory.py:453-455.  hsru_delta_cuda.pkm_fused_forward chains it with the PKM
recurrence.

`dense_route` is the counterpart of _route_dense's slot-projection branch
(memory.py:233-236) with the q_scale multiply of memory.py:490-492, one tcgen05
kernel (dg_dense_route); hsru_delta_cuda.dense_fused_forward chains it with the
dense recurrence.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

from . import _lib

_DT = {torch.float32: 0, torch.float64: 1, torch.float16: 2, torch.bfloat16: 3}


def pkm_route(k: torch.Tensor, q: torch.Tensor, router_k: Sequence[torch.Tensor],
              router_q: Sequence[torch.Tensor], top_k: int,
              q_scale: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """k, q [B,H,T,Dh] -> (wk, wq, idx) [B,H,T,top_k**2]; router weights [G_a, Dh] fp32."""
    if not (k.is_cuda and q.is_cuda):
        raise RuntimeError("k and q must be CUDA tensors")
    if len(router_k) != 2 or len(router_q) != 2:
        raise RuntimeError("pkm_route handles two routing axes")
    k_c, q_c = k.contiguous(), q.contiguous().to(k.dtype)
    wts = [w.detach().to(device=k.device, dtype=torch.float32).contiguous() for w in (*router_k, *router_q)]
    qs = q_scale.detach().to(device=k.device, dtype=torch.float32).contiguous() if q_scale is not None else None
    B, H, T, Dh = k_c.shape
    A = top_k * top_k
    wk = torch.empty((B, H, T, A), dtype=k_c.dtype, device=k.device)
    wq = torch.empty_like(wk)
    idx = torch.empty((B, H, T, A), dtype=torch.int64, device=k.device)
    with torch.cuda.device(k.device):
        _lib.call("dg_pkm_route", _DT[k_c.dtype], B, H, T, Dh, wts[0].shape[0], wts[1].shape[0], top_k,
                  k_c.data_ptr(), q_c.data_ptr(), *(w.data_ptr() for w in wts),
                  qs.data_ptr() if qs is not None else None, wk.data_ptr(), wq.data_ptr(), idx.data_ptr(),
                  torch.cuda.current_stream(k.device).cuda_stream)
    return wk, wq, idx


def dense_route_covers(k: torch.Tensor, slot_proj_k: torch.Tensor) -> bool:
    """Whether dg_dense_route takes this call: 16-bit CUDA keys, Dh = 64, slots a
    multiple of 64 up to 512."""
    S = slot_proj_k.shape[0]
    return (k.is_cuda and k.dtype in (torch.float16, torch.bfloat16) and k.shape[-1] == 64
            and slot_proj_k.shape[-1] == 64 and S % 64 == 0 and 64 <= S <= 512)


def dense_route(k: torch.Tensor, q: torch.Tensor, slot_proj_k: torch.Tensor, slot_proj_q: torch.Tensor,
                q_scale: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """k, q [B,H,T,64] (f16 / bf16) -> wk = normalize(k P_k^T), wq = (q P_q^T) q_scale[h],
    each [B,H,T,slots] in k's dtype; P_* [slots, 64] (the layer's nn.Linear weights)."""
    if not dense_route_covers(k, slot_proj_k):
        raise RuntimeError("dense_route: needs 16-bit CUDA k, q with Dh = 64 and slots a multiple of 64 up to 512")
    from . import _hsru
    k_c, q_c = k.contiguous(), q.contiguous().to(k.dtype)
    pk = slot_proj_k.detach().to(device=k.device, dtype=k.dtype).contiguous()
    pq = slot_proj_q.detach().to(device=k.device, dtype=k.dtype).contiguous()
    qs = q_scale.detach().to(device=k.device, dtype=torch.float32).contiguous() if q_scale is not None else None
    B, H, T, Dh = k_c.shape
    S = pk.shape[0]
    wk = torch.empty((B, H, T, S), dtype=k_c.dtype, device=k.device)
    wq = torch.empty_like(wk)
    index = k.device.index if k.device.index is not None else torch.cuda.current_device()
    status = _hsru.device_status_word(index)
    with torch.cuda.device(k.device):
        _lib.call("dg_dense_route", _DT[k_c.dtype], B, H, T, Dh, S, k_c.data_ptr(), q_c.data_ptr(), pk.data_ptr(),
                  pq.data_ptr(), qs.data_ptr() if qs is not None else None, wk.data_ptr(), wq.data_ptr(),
                  status.data_ptr(), torch.cuda.current_stream(k.device).cuda_stream)
    return wk, wq
