"""Drop-in replacement for the reference torch extension ``hsru_delta_cuda``.

Same functions, argument names, defaults, return lists and error behaviour as
the reference pybind module (src/cpp/binding.cpp:523-561).  The six functions
are the compiled extension ``deltagrid_b200._hsru`` (csrc/binding.cpp): each
checks and prepares its tensors as the reference binding does, allocates its
outputs with torch's caching allocator and calls one entry point of the C ABI
(include/deltagrid_b200.h) on torch's current CUDA stream of the input's device.

Install it under the reference's module name with ``deltagrid_b200.install()``
(or put the repository root on sys.path: ``hsru_delta_cuda.py`` there
re-exports this module); the reference loader (src/ops/_backend.py:31-37)
then picks it up with no change to the reference layer.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.nn.functional as F

from . import _lib

try:
    from . import _hsru
except ImportError as e:     # no CPU fallback: the compiled module is the product
    raise ImportError("deltagrid_b200._hsru (the compiled hsru_delta_cuda binding) is not built or does not "
                      "load; build it with `python -m deltagrid_b200.build`") from e

# forward(q, k, v, beta, wk, wq, decay, s_init=None, save_for_backward=False, algo=0)
#   -> [out, s_final, err_out, s_final_f]                         (binding.cpp:36-113)
forward = _hsru.forward
# step(q, k, v, beta, wk, wq, decay, s_prev) -> [out, s_next]     (binding.cpp:130-203)
step = _hsru.step
# pkm_step(v, beta, wk, wq, active_idx, decay, state_1m) -> [out, state]   (binding.cpp:319-370)
pkm_step = _hsru.pkm_step
# pkm_forward(v, beta, wk, wq, active_idx, decay, state, save_for_backward=False)
#   -> [out, state, saved_s_act]                                  (binding.cpp:375-434)
pkm_forward = _hsru.pkm_forward
# pkm_forward with an explicit kernel (dg_pkm_algo); raises DeltaGridError if it does not cover the call
pkm_forward_algo = _hsru.pkm_forward_algo
# backward(grad_out, grad_s_final, v, beta, wk, wq, decay, s_final, err_saved, needs_grad_s_init=False)
#   -> [grad_v, grad_beta, grad_wk, grad_wq, grad_decay, grad_s_init]      (binding.cpp:223-312)
backward = _hsru.backward
# pkm_backward(grad_out, v, beta, wk, wq, active_idx, decay, saved_s_act, total_slots,
#              grad_final_state=None, needs_grad_decay=False)
#   -> [grad_v, grad_beta, grad_wk, grad_wq, grad_decay, grad_state]       (binding.cpp:439-518)
pkm_backward = _hsru.pkm_backward


def device_status(device=None, clear: bool = True) -> int:
    """Synchronizes and returns the kernel self-check bits recorded on ``device``.

    Bit 0x1 (DG_DEVCHK_INDEX_RANGE) means a PKM slot index was outside
    [0, total_slots): that row was skipped.  Bit 0x4 (DG_DEVCHK_TIMEOUT) means a
    bounded wait inside a kernel gave up: that launch's results are invalid.
    """
    device = torch.device(device if device is not None else torch.cuda.current_device())
    if device.type != "cuda":
        device = torch.device("cuda", device.index or 0)
    index = device.index if device.index is not None else torch.cuda.current_device()
    w = _hsru.device_status_word(index)
    val = int(w.item())
    if clear:
        w.zero_()
    return val


def set_wait_limit(polls: int) -> int:
    """Sets the poll budget of the kernels' bounded waits (dg_set_wait_limit) and returns
    the previous one.  0 makes every such wait give up at once: the launch then flags
    DG_DEVCHK_TIMEOUT (0x4) in device_status() and its results are invalid."""
    return int(_lib.lib().dg_set_wait_limit(int(polls)))


def pkm_fused_forward(k: torch.Tensor, q: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                      router_k, router_q, q_scale: Optional[torch.Tensor], decay: torch.Tensor,
                      state: torch.Tensor, top_k: int = 8, grid=None,
                      save: bool = False) -> List[Optional[torch.Tensor]]:
    """Routing plus recurrence: what DeltaGridLayer.forward does in Sparse Delta-PKM
    mode between its projections and out_proj (memory.py:452-464 then :510).

    k, q [B,H,T,Dh]; router_k / router_q two [G_a, Dh] weights each (the layer's
    axes_proj_k / axes_proj_q); q_scale [H] or None.  Returns [out, state, idx,
    saved_s_act]; state is updated in place as in pkm_forward.
    """
    from .route import pkm_route
    if grid is not None and tuple(grid) != (router_k[0].shape[0], router_k[1].shape[0]):
        raise RuntimeError(f"pkm_fused_forward: grid {tuple(grid)} does not match the router weights")
    wk, wq, idx = pkm_route(k, q, router_k, router_q, top_k, q_scale)
    out, state_c, saved = pkm_forward(v, beta, wk, wq, idx, decay, state, save)
    return [out, state_c, idx, saved]


def dense_fused_forward(k: torch.Tensor, q: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                        slot_proj_k: Optional[torch.Tensor], slot_proj_q: Optional[torch.Tensor],
                        q_scale: Optional[torch.Tensor], decay: torch.Tensor, s_init: Optional[torch.Tensor] = None,
                        save_for_backward: bool = False) -> List[torch.Tensor]:
    """Slot routing plus recurrence: what DeltaGridLayer.forward does in dense mode
    between its projections and out_proj (memory.py:488-512).

    k, q, v [B,H,T,Dh]; beta [B,H,T]; slot_proj_k / slot_proj_q [slots, Dh] (the
    layer's nn.Linear weights) or None when slots == Dh; q_scale [H] or None.
    wk = L2-normalise(k P_k^T) and wq = (q P_q^T) q_scale (memory.py:233-236,
    :490-492), formed by the slot-routing kernel (route.dense_route: 16-bit k, Dh = 64,
    slots a multiple of 64 up to 512; other shapes use torch's GEMMs) and kept in HBM
    for the recurrence kernel; returns forward's [out, s_final, err_out, s_final_f].
    """
    from .route import dense_route, dense_route_covers
    if (slot_proj_k is None) != (slot_proj_q is None):
        raise RuntimeError("dense_fused_forward: give both slot projections or neither")
    if slot_proj_k is not None and dense_route_covers(k, slot_proj_k):
        wk, wq = dense_route(k, q, slot_proj_k, slot_proj_q, q_scale)
    else:
        if slot_proj_k is not None:
            wk = F.normalize(F.linear(k, slot_proj_k.to(k.dtype)), p=2, dim=-1)
            wq = F.linear(q, slot_proj_q.to(q.dtype))
        else:
            wk, wq = k, q
        if q_scale is not None:
            wq = wq * q_scale.to(dtype=q.dtype).view(1, -1, 1, 1)
    return forward(q, k, v, beta, wk, wq, decay, s_init, save_for_backward)


__all__ = ["forward", "step", "pkm_step", "pkm_forward", "pkm_forward_algo", "backward", "pkm_backward",
           "device_status", "set_wait_limit", "pkm_fused_forward", "dense_fused_forward", "DeltaGridError"]

DeltaGridError = _lib.DeltaGridError
