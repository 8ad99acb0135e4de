"""Drop-in replacement for the reference torch extension ``hsru_delta_cuda``.

Same functions, argument names, defaults, return lists and error behaviour as
the reference pybind module (src/cpp/binding.cpp:523-561); the work is done by
the sm_100a kernels behind the C ABI (include/deltagrid_b200.h), launched on
torch's current CUDA stream of the input's device.  Outputs are allocated with
torch (the caching allocator), as the reference binding does.

Install it under the reference's module name with ``deltagrid_b200.install()``
(or put the repository root on sys.path: ``hsru_delta_cuda.py`` there
re-exports this module); the reference loader (src/ops/_backend.py:31-37)
then picks it up with no change to the reference layer.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from . import _lib

_DT = {torch.float32: _lib.DTYPE_F32, torch.float64: _lib.DTYPE_F64,
       torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}

_status_words = {}


def _check_cuda(t: torch.Tensor, name: str) -> None:
    # binding.cpp:18 -- TORCH_CHECK(x.is_cuda(), #x " must be a CUDA tensor")
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")


def _dtype_code(t: torch.Tensor, op: str) -> int:
    code = _DT.get(t.dtype)
    if code is None:
        # AT_DISPATCH_FLOATING_TYPES_AND2 error for other dtypes (binding.cpp:90-92)
        raise RuntimeError(f'"{op}" not implemented for \'{str(t.dtype).replace("torch.", "")}\'')
    return code


def _same_dtype(ref: torch.Tensor, op: str, **ts) -> None:
    # data_ptr<scalar_t>() in the reference raises on a dtype mismatch
    for name, t in ts.items():
        if t is not None and t.dtype != ref.dtype:
            raise RuntimeError(f"{op}: expected {name} to have dtype {ref.dtype}, got {t.dtype}")


def _contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(t: torch.Tensor) -> int:
    # the caller's current stream on t's device (the raw handle: no Stream object)
    if _raw_stream is not None:
        return _raw_stream(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


class _on_device:
    """`with torch.cuda.device(d)` only when d is not already current: switching the
    device costs more host time than a decode step's kernel takes."""
    __slots__ = ("idx", "ctx")

    def __init__(self, device: torch.device):
        self.idx = device.index
        self.ctx = None

    def __enter__(self):
        if self.idx is not None and self.idx != torch.cuda.current_device():
            self.ctx = torch.cuda.device(self.idx)
            self.ctx.__enter__()
        return self

    def __exit__(self, *exc):
        if self.ctx is not None:
            self.ctx.__exit__(*exc)
        return False


def _status_word(device: torch.device) -> torch.Tensor:
    w = _status_words.get(device)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=device)
        _status_words[device] = w
    return w


def device_status(device=None, clear: bool = True) -> int:
    """Synchronizes and returns the kernel self-check bits recorded on ``device``.

    Bit 0x1 (DG_DEVCHK_INDEX_RANGE) means a PKM slot index was outside
    [0, total_slots): that row was skipped.
    """
    device = torch.device(device if device is not None else torch.cuda.current_device())
    if device.type != "cuda":
        device = torch.device("cuda", device.index or 0)
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    w = _status_word(device)
    val = int(w.item())
    if clear:
        w.zero_()
    return val


def forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
            wk: torch.Tensor, wq: torch.Tensor, decay: torch.Tensor,
            s_init: Optional[torch.Tensor] = None, save_for_backward: bool = False,
            algo: int = _lib.ALGO_AUTO) -> List[Optional[torch.Tensor]]:
    """Dense sequence forward (binding.cpp:36-113).

    Returns [out, s_final, err_out, s_final_f]; err_out (fp32 residuals) is None
    unless save_for_backward; s_final_f is an fp32 copy of the final state when
    saving for a non-fp32 dtype, else the s_final tensor itself.
    """
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (beta, "beta"), (wk, "wk"), (wq, "wq"), (decay, "decay")):
        _check_cuda(t, n)
    v_c, beta_c, wk_c, wq_c, decay_c = map(_contig, (v, beta, wk, wq, decay))
    code = _dtype_code(v_c, "delta_grid_forward_cuda")
    _same_dtype(v_c, "forward", beta=beta_c, wk=wk_c, wq=wq_c, decay=decay_c)
    B, H, T, Dh = v_c.shape
    slots = wk_c.size(3)
    has_init = s_init is not None
    s_init_c = None
    if has_init:
        _check_cuda(s_init, "s_init.value()")
        s_init_c = _contig(s_init)
        _same_dtype(v_c, "forward", s_init=s_init_c)
    out = torch.empty((B, H, T, Dh), dtype=v_c.dtype, device=v_c.device)
    s_final = torch.empty((B, H, slots, Dh), dtype=v_c.dtype, device=v_c.device)
    is_fp32 = v_c.dtype == torch.float32
    err_out = torch.empty((B, H, T, Dh), dtype=torch.float32, device=v_c.device) if save_for_backward else None
    s_final_f = (torch.empty((B, H, slots, Dh), dtype=torch.float32, device=v_c.device)
                 if (save_for_backward and not is_fp32) else s_final)
    dynamic = 1 if decay_c.dim() > 1 else 0
    with _on_device(v_c.device):
        _lib.call("dg_dense_forward_ex", code, B, H, T, slots, Dh, v_c.data_ptr(), beta_c.data_ptr(),
                  wk_c.data_ptr(), wq_c.data_ptr(), decay_c.data_ptr(), dynamic,
                  s_init_c.data_ptr() if has_init else None, out.data_ptr(), s_final.data_ptr(),
                  err_out.data_ptr() if err_out is not None else None,
                  s_final_f.data_ptr() if (save_for_backward and not is_fp32) else None,
                  int(algo), _stream(v_c))
    return [out, s_final, err_out, s_final_f]


def step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
         wk: torch.Tensor, wq: torch.Tensor, decay: torch.Tensor,
         s_prev: torch.Tensor) -> List[torch.Tensor]:
    """Single decode step (binding.cpp:130-203).  Returns [out, s_next].

    v, wk, wq and beta may be strided over (batch, head) when their last
    dimension is contiguous; outputs take q's dtype and device, as in the reference.
    """
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (beta, "beta"), (wk, "wk"), (wq, "wq"),
                 (decay, "decay"), (s_prev, "s_prev")):
        _check_cuda(t, n)
    v_c = v if v.stride(2) == 1 else v.contiguous()
    wk_c = wk if wk.stride(2) == 1 else wk.contiguous()
    wq_c = wq if wq.stride(2) == 1 else wq.contiguous()
    dynamic = decay.dim() > 1
    decay_c = decay.contiguous() if (not dynamic and decay.stride(0) != 1) else decay
    s_prev_c = _contig(s_prev)
    code = _dtype_code(v_c, "delta_grid_step_cuda")
    _same_dtype(v_c, "step", beta=beta, wk=wk_c, wq=wq_c, decay=decay_c, s_prev=s_prev_c)
    B, H, Dh = v_c.shape
    slots = wk_c.size(2)
    out = torch.empty((B, H, Dh), dtype=q.dtype, device=q.device)
    s_next = torch.empty((B, H, slots, Dh), dtype=q.dtype, device=q.device)
    _same_dtype(v_c, "step", out=out)
    d_sb, d_sh = (decay_c.stride(0), decay_c.stride(1)) if dynamic else (0, 1)
    vs, bs, ks, qs = v_c.stride(), beta.stride(), wk_c.stride(), wq_c.stride()
    with _on_device(v_c.device):
        _lib.check(_lib.fn("dg_dense_step")(code, B, H, slots, Dh, v_c.data_ptr(), vs[0], vs[1],
                                            beta.data_ptr(), bs[0], bs[1], wk_c.data_ptr(), ks[0], ks[1],
                                            wq_c.data_ptr(), qs[0], qs[1], decay_c.data_ptr(), int(dynamic),
                                            d_sb, d_sh, s_prev_c.data_ptr(), out.data_ptr(), s_next.data_ptr(),
                                            _stream(v_c)), "dg_dense_step")
    return [out, s_next]


def pkm_step(v: torch.Tensor, beta: torch.Tensor, wk: torch.Tensor, wq: torch.Tensor,
             active_idx: torch.Tensor, decay: torch.Tensor, state_1m: torch.Tensor) -> List[torch.Tensor]:
    """Sparse Delta-PKM decode step, state updated in place (binding.cpp:319-370).

    Returns [out, state].  A [B,H] decay is applied per batch row (the PyTorch
    path's semantics, memory.py:582-591).
    """
    for t, n in ((v, "v"), (beta, "beta"), (wk, "wk"), (wq, "wq"), (active_idx, "active_idx"),
                 (decay, "decay"), (state_1m, "state_1m")):
        _check_cuda(t, n)
    v_c, beta_c, wk_c, wq_c, idx_c, decay_c = map(_contig, (v, beta, wk, wq, active_idx, decay))
    state_c = _contig(state_1m)
    code = _dtype_code(v_c, "delta_pkm_step_cuda")
    _same_dtype(v_c, "pkm_step", beta=beta_c, wk=wk_c, wq=wq_c, decay=decay_c, state=state_c)
    if idx_c.dtype != torch.int64:
        raise RuntimeError(f"pkm_step: expected active_idx to have dtype torch.int64, got {idx_c.dtype}")
    B, H, Dh = v_c.shape
    A = wk_c.size(2)
    total = state_c.size(2)
    out = torch.empty((B, H, Dh), dtype=v_c.dtype, device=v_c.device)
    dynamic = 1 if decay_c.dim() > 1 else 0
    with _on_device(v_c.device):
        _lib.call("dg_pkm_step", code, B, H, A, total, Dh, v_c.data_ptr(), beta_c.data_ptr(),
                  wk_c.data_ptr(), wq_c.data_ptr(), idx_c.data_ptr(), decay_c.data_ptr(), dynamic,
                  state_c.data_ptr(), out.data_ptr(), _status_word(v_c.device).data_ptr(),
                  _stream(v_c))
    return [out, state_c]


def pkm_forward(v: torch.Tensor, beta: torch.Tensor, wk: torch.Tensor, wq: torch.Tensor,
                active_idx: torch.Tensor, decay: torch.Tensor, state: torch.Tensor,
                save_for_backward: bool = False) -> List[Optional[torch.Tensor]]:
    """Sparse Delta-PKM sequence forward, state updated in place (binding.cpp:375-434).

    Returns [out, state, saved_s_act]; saved_s_act [B,H,T,A,Dh] holds the rows
    gathered at each step when save_for_backward, else None.
    """
    return pkm_forward_algo(v, beta, wk, wq, active_idx, decay, state, save_for_backward, _lib.PKM_AUTO)


def pkm_forward_algo(v: torch.Tensor, beta: torch.Tensor, wk: torch.Tensor, wq: torch.Tensor,
                     active_idx: torch.Tensor, decay: torch.Tensor, state: torch.Tensor,
                     save_for_backward: bool = False, algo: int = 0) -> List[Optional[torch.Tensor]]:
    """pkm_forward with an explicit kernel (dg_pkm_algo); raises if it does not cover the call."""
    for t, n in ((v, "v"), (beta, "beta"), (wk, "wk"), (wq, "wq"), (active_idx, "active_idx"),
                 (decay, "decay"), (state, "state")):
        _check_cuda(t, n)
    v_c, beta_c, wk_c, wq_c, idx_c, decay_c = map(_contig, (v, beta, wk, wq, active_idx, decay))
    state_c = _contig(state)
    code = _dtype_code(v_c, "delta_pkm_forward_cuda")
    _same_dtype(v_c, "pkm_forward", beta=beta_c, wk=wk_c, wq=wq_c, decay=decay_c, state=state_c)
    if idx_c.dtype != torch.int64:
        raise RuntimeError(f"pkm_forward: expected active_idx to have dtype torch.int64, got {idx_c.dtype}")
    B, H, T, Dh = v_c.shape
    A = wk_c.size(3)
    total = state_c.size(2)
    out = torch.empty((B, H, T, Dh), dtype=v_c.dtype, device=v_c.device)
    saved = (torch.empty((B, H, T, A, Dh), dtype=v_c.dtype, device=v_c.device)
             if save_for_backward else None)
    dynamic = 1 if decay_c.dim() > 1 else 0
    with _on_device(v_c.device):
        # scratch for kernels that need it (per-row hazard codes), from torch's caching allocator
        nws = _lib.lib().dg_pkm_forward_workspace_size(code, B, H, T, A, total, Dh, int(algo))
        ws = torch.empty(nws, dtype=torch.uint8, device=v_c.device) if nws else None
        _lib.call("dg_pkm_forward_ex", code, B, H, T, A, total, Dh, v_c.data_ptr(), beta_c.data_ptr(),
                  wk_c.data_ptr(), wq_c.data_ptr(), idx_c.data_ptr(), decay_c.data_ptr(), dynamic,
                  state_c.data_ptr(), out.data_ptr(), saved.data_ptr() if saved is not None else None,
                  _status_word(v_c.device).data_ptr(), int(algo), ws.data_ptr() if ws is not None else None,
                  nws, _stream(v_c))
    return [out, state_c, saved]


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


def backward(grad_out: torch.Tensor, grad_s_final: Optional[torch.Tensor], v: torch.Tensor,
             beta: torch.Tensor, wk: torch.Tensor, wq: torch.Tensor, decay: torch.Tensor,
             s_final: torch.Tensor, err_saved: torch.Tensor,
             needs_grad_s_init: bool = False) -> List[Optional[torch.Tensor]]:
    """Dense analytic backward (binding.cpp:223-312).

    s_final and err_saved are the fp32 final state and residuals of forward(...,
    save_for_backward=True) (its s_final_f / err_out).  Returns [grad_v, grad_beta,
    grad_wk, grad_wq, grad_decay, grad_s_init]; grad_s_init is an undefined (None)
    tensor unless needs_grad_s_init.  A static [H] decay gets the sum over the batch.
    """
    for t, n in ((grad_out, "grad_out"), (v, "v"), (beta, "beta"), (wk, "wk"), (wq, "wq"), (decay, "decay"),
                 (s_final, "s_final"), (err_saved, "err_saved")):
        _check_cuda(t, n)
    go_c, v_c, beta_c, wk_c, wq_c, decay_c = map(_contig, (grad_out, v, beta, wk, wq, decay))
    sf_c = s_final.to(torch.float32).contiguous()
    err_c = err_saved.to(torch.float32).contiguous()
    code = _dtype_code(v_c, "delta_grid_backward_cuda")
    _same_dtype(v_c, "backward", grad_out=go_c, beta=beta_c, wk=wk_c, wq=wq_c, decay=decay_c)
    B, H, T, Dh = v_c.shape
    S = wk_c.size(3)
    gsf = None
    if grad_s_final is not None:
        _check_cuda(grad_s_final, "grad_s_final")
        gsf = _contig(grad_s_final)
        _same_dtype(v_c, "backward", grad_s_final=gsf)
    dynamic = 1 if decay_c.dim() > 1 else 0
    grad_v = torch.empty_like(v_c)
    grad_beta = torch.empty_like(beta_c)
    grad_wk = torch.empty_like(wk_c)
    grad_wq = torch.empty_like(wq_c)
    grad_decay = torch.empty_like(decay_c) if dynamic else torch.zeros_like(decay_c)
    grad_s_init = torch.empty((B, H, S, Dh), dtype=v_c.dtype, device=v_c.device) if needs_grad_s_init else None
    with _on_device(v_c.device):
        nws = _lib.lib().dg_dense_backward_workspace_size(B, H, S, Dh)
        ws = torch.empty(nws // 4, dtype=torch.float32, device=v_c.device) if nws else None
        _lib.call("dg_dense_backward", code, B, H, T, S, Dh, go_c.data_ptr(),
                  gsf.data_ptr() if gsf is not None else None, v_c.data_ptr(), beta_c.data_ptr(),
                  wk_c.data_ptr(), wq_c.data_ptr(), decay_c.data_ptr(), dynamic, sf_c.data_ptr(), err_c.data_ptr(),
                  grad_v.data_ptr(), grad_beta.data_ptr(), grad_wk.data_ptr(), grad_wq.data_ptr(),
                  grad_decay.data_ptr(), grad_s_init.data_ptr() if grad_s_init is not None else None,
                  ws.data_ptr() if ws is not None else None, _stream(v_c))
    return [grad_v, grad_beta, grad_wk, grad_wq, grad_decay, grad_s_init]


def pkm_backward(grad_out: torch.Tensor, v: torch.Tensor, beta: torch.Tensor, wk: torch.Tensor,
                 wq: torch.Tensor, active_idx: torch.Tensor, decay: torch.Tensor, saved_s_act: torch.Tensor,
                 total_slots: int, grad_final_state: Optional[torch.Tensor] = None,
                 needs_grad_decay: bool = False) -> List[Optional[torch.Tensor]]:
    """Sparse Delta-PKM analytic backward (binding.cpp:439-518).

    saved_s_act is the [B,H,T,A,Dh] rows of pkm_forward(..., save_for_backward=True).
    Returns [grad_v, grad_beta, grad_wk, grad_wq, grad_decay, grad_state]: grad_state
    is the gradient of the initial state (grad_final_state carried back to step 0),
    grad_decay is None unless needs_grad_decay ([B,H,T] for a dynamic decay, else [H]
    summed over the batch -- an output the reference allocates but never writes).
    """
    for t, n in ((grad_out, "grad_out"), (v, "v"), (beta, "beta"), (wk, "wk"), (wq, "wq"),
                 (active_idx, "active_idx"), (decay, "decay"), (saved_s_act, "saved_s_act")):
        _check_cuda(t, n)
    go_c, v_c, beta_c, wk_c, wq_c, idx_c, decay_c, sv_c = map(
        _contig, (grad_out, v, beta, wk, wq, active_idx, decay, saved_s_act))
    code = _dtype_code(v_c, "delta_pkm_backward_cuda")
    _same_dtype(v_c, "pkm_backward", grad_out=go_c, beta=beta_c, wk=wk_c, wq=wq_c, decay=decay_c,
                saved_s_act=sv_c)
    if idx_c.dtype != torch.int64:
        raise RuntimeError(f"pkm_backward: expected active_idx to have dtype torch.int64, got {idx_c.dtype}")
    B, H, T, Dh = v_c.shape
    A = wk_c.size(3)
    total = int(total_slots)
    dynamic = 1 if decay_c.dim() > 1 else 0
    if grad_final_state is not None:
        _check_cuda(grad_final_state, "grad_final_state")
        grad_state = grad_final_state.clone().contiguous()
        _same_dtype(v_c, "pkm_backward", grad_final_state=grad_state)
    else:
        grad_state = torch.zeros((B, H, total, Dh), dtype=v_c.dtype, device=v_c.device)
    grad_v = torch.empty((B, H, T, Dh), dtype=v_c.dtype, device=v_c.device)
    grad_beta = torch.empty((B, H, T), dtype=v_c.dtype, device=v_c.device)
    grad_wk = torch.empty((B, H, T, A), dtype=v_c.dtype, device=v_c.device)
    grad_wq = torch.empty((B, H, T, A), dtype=v_c.dtype, device=v_c.device)
    grad_decay = None
    if needs_grad_decay:
        grad_decay = (torch.empty((B, H, T), dtype=v_c.dtype, device=v_c.device) if dynamic
                      else torch.zeros((H,), dtype=v_c.dtype, device=v_c.device))
    with _on_device(v_c.device):
        _lib.call("dg_pkm_backward", code, B, H, T, A, total, Dh, go_c.data_ptr(), v_c.data_ptr(),
                  beta_c.data_ptr(), wk_c.data_ptr(), wq_c.data_ptr(), idx_c.data_ptr(), decay_c.data_ptr(),
                  dynamic, sv_c.data_ptr(), grad_state.data_ptr(), grad_v.data_ptr(), grad_beta.data_ptr(),
                  grad_wk.data_ptr(), grad_wq.data_ptr(), grad_decay.data_ptr() if grad_decay is not None else None,
                  _status_word(v_c.device).data_ptr(), _stream(v_c))
    return [grad_v, grad_beta, grad_wk, grad_wq, grad_decay, grad_state]
