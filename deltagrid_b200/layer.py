"""DeltaGridLayer on this package's kernels: the reference layer's parameters, forward
and step API (src/modules/memory.py:49-638), with the recurrence on the B200 path.

The parameters have the reference's names and shapes, so a state_dict moves between
the two layers unchanged.  What differs is how the recurrence is reached:

* Inference (autograd off, or nothing that needs a gradient): Sparse Delta-PKM runs
  the fused two-axis router (dg_pkm_route, the routing of memory.py:240-289 and the
  q_scale of :453-455) and then the sequence kernel on the caller's state IN PLACE:
  the state tensor passed in is updated and returned.  No copy of the state, no
  compaction of the touched slots and no per-step saved rows are made, where the
  reference's autograd function (src/ops/_autograd.py:88-177) clones the state (or
  runs torch.unique over every index) and saves [B,H,T,64,Dh] rows on every call --
  about 69 GB at the 1024 x 1024 grid's bench shape.  Dense mode with slot
  projections on 16-bit keys (Dh = 64, slots a multiple of 64 up to 512) forms wk and
  wq with the slot-routing kernel (dg_dense_route: memory.py:233-236 and the q_scale
  of :490-492), then calls the sequence forward with the state as s_init and returns
  the new state.
* Training: autograd functions over this package's forward (saving what its backward
  needs) and backward kernels.  The PKM one runs on a copy of the touched slots of
  the state, so the caller's state is left as it was, as in the reference.

Modes: standard dense (slots >= Dh), factorized Kronecker dense (grid_dim without
top_k; routed in torch as memory.py:219-231 does), Sparse Delta-PKM (grid_dim and
top_k; two axes without subspace slicing use the fused router, other shapes route
in torch).
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import hsru_delta_cuda as ext
from .route import dense_route, dense_route_covers, pkm_route


class _DenseRecurrence(torch.autograd.Function):
    """y, S_T = dense recurrence(v, beta, wk, wq, decay, S_0); gradients by dg_dense_backward."""

    @staticmethod
    def forward(ctx, q, v, beta, wk, wq, decay, s_init):
        out, s_final, err, s_final_f = ext.forward(q, v, v, beta, wk, wq, decay, s_init, True)
        ctx.save_for_backward(v, beta, wk, wq, decay, s_final_f, err)
        ctx.want_s_init = s_init is not None and s_init.requires_grad
        return out, s_final

    @staticmethod
    def backward(ctx, g_out, g_s):
        v, beta, wk, wq, decay, s_final_f, err = ctx.saved_tensors
        g_out = g_out.to(v.dtype).contiguous()
        g_s = g_s.to(v.dtype).contiguous() if g_s is not None else None
        gv, gb, gwk, gwq, gd, gs0 = ext.backward(g_out, g_s, v, beta, wk, wq, decay, s_final_f, err, ctx.want_s_init)
        return None, gv, gb, gwk, gwq, gd, (gs0 if ctx.want_s_init else None)


class _PkmRecurrence(torch.autograd.Function):
    """PKM recurrence for training.  The kernel runs on a compact copy of the slots the
    sequence touches (or of the whole state when that is small), so the input state is
    left unchanged; the rows each step read are saved for dg_pkm_backward."""

    @staticmethod
    def forward(ctx, v, beta, wk, wq, idx, decay, state):
        B, H, T, Dh = v.shape
        total = state.shape[2]
        compact = total > 4096 and total > idx.shape[-1] * T
        if compact:
            slots, run_idx = torch.unique(idx, return_inverse=True)
            sel = slots.view(1, 1, -1, 1).expand(B, H, slots.numel(), Dh)
            work = torch.gather(state, 2, sel).contiguous()
        else:
            slots, run_idx, sel = None, idx, None
            work = state.clone()
        out, work, saved = ext.pkm_forward(v, beta, wk, wq, run_idx.contiguous(), decay, work, True)
        if compact:
            final = state.clone().scatter_(2, sel, work)
        else:
            final = work
        ctx.save_for_backward(v, beta, wk, wq, run_idx, decay, saved)
        ctx.sel, ctx.n_work, ctx.total, ctx.compact = sel, work.shape[2], total, compact
        return out, final

    @staticmethod
    def backward(ctx, g_out, g_state):
        v, beta, wk, wq, run_idx, decay, saved = ctx.saved_tensors
        g_fin = None
        if g_state is not None:
            g_fin = (torch.gather(g_state, 2, ctx.sel) if ctx.compact else g_state).to(v.dtype).contiguous()
        need_decay = ctx.needs_input_grad[5]
        gv, gb, gwk, gwq, gd, gs = ext.pkm_backward(g_out.to(v.dtype).contiguous(), v, beta, wk, wq, run_idx, decay,
                                                    saved, ctx.n_work, g_fin, need_decay)
        g_init = None
        if ctx.needs_input_grad[6]:
            if ctx.compact:
                g_init = (g_state.clone() if g_state is not None else
                          torch.zeros(v.shape[0], v.shape[1], ctx.total, v.shape[3], device=v.device, dtype=v.dtype))
                g_init.scatter_(2, ctx.sel, gs)
            else:
                g_init = gs
        return gv, gb, gwk, gwq, None, (gd if need_decay else None), g_init


class DeltaGridLayer(nn.Module):
    """Drop-in for the reference DeltaGridLayer (src/modules/memory.py:30-638) on CUDA
    tensors.  Constructor arguments as the reference's; a config object with the same
    attribute names may be passed as ``config``."""

    def __init__(self, d_model: Optional[int] = None, num_heads: int = 4, num_slots: Optional[int] = None,
                 grid_dim: Optional[Sequence[int]] = None, top_k: Optional[int] = None, decay_init: float = 1.0,
                 dynamic_decay: bool = True, strict_slots: bool = False, use_chunkwise: bool = False,
                 chunk_size: int = 64, subspace_slicing: bool = False, config=None):
        super().__init__()
        if config is not None:
            d_model, num_heads, num_slots = config.d_model, config.num_heads, config.num_slots
            grid_dim, top_k, decay_init = config.grid_dim, config.top_k, config.decay_init
            dynamic_decay, strict_slots = config.dynamic_decay, config.strict_slots
            use_chunkwise, chunk_size = config.use_chunkwise, config.chunk_size
            subspace_slicing = getattr(config, "subspace_slicing", False)
        dim = int(d_model if d_model is not None else 128)
        if dim % num_heads:
            raise ValueError(f"d_model ({dim}) must be divisible by num_heads ({num_heads})")
        if top_k is not None and grid_dim is None:
            raise ValueError("top_k was specified without grid_dim")
        self.d_model, self.num_heads, self.head_dim = dim, num_heads, dim // num_heads
        self.grid_dim = tuple(grid_dim) if grid_dim is not None else None
        self.top_k = top_k
        self.dynamic_decay = dynamic_decay
        self.use_chunkwise = use_chunkwise
        self.chunk_size = chunk_size
        self.subspace_slicing = bool(subspace_slicing and self.grid_dim is not None
                                     and self.head_dim % len(self.grid_dim) == 0)
        self.slice_dim = self.head_dim // len(self.grid_dim) if self.subspace_slicing else self.head_dim

        # parameters: names, shapes and initialisation of memory.py:135-226
        self.proj_qkv_beta = nn.Linear(dim, 3 * dim + num_heads, bias=False)
        with torch.no_grad():
            w = self.proj_qkv_beta.weight
            for i in range(3):
                nn.init.orthogonal_(w[i * dim:(i + 1) * dim])
            nn.init.zeros_(w[3 * dim:])
        self.axes_proj_k = self.axes_proj_q = None
        self.slot_proj_k = self.slot_proj_q = None
        if self.grid_dim is not None:
            in_dim = self.slice_dim if top_k is not None else self.head_dim
            self.total_slots = math.prod(self.grid_dim)
            self.active_slots = top_k ** len(self.grid_dim) if top_k is not None else self.total_slots
            self.num_slots = self.actual_slots = self.total_slots
            self.axes_proj_k = nn.ModuleList([nn.Linear(in_dim, g, bias=False) for g in self.grid_dim])
            self.axes_proj_q = nn.ModuleList([nn.Linear(in_dim, g, bias=False) for g in self.grid_dim])
            for pk, pq in zip(self.axes_proj_k, self.axes_proj_q):
                nn.init.orthogonal_(pk.weight)
                with torch.no_grad():
                    pq.weight.copy_(pk.weight)
        else:
            self.num_slots = self.head_dim if num_slots is None else num_slots
            self.actual_slots = (num_slots if (strict_slots and num_slots is not None)
                                 else max(self.num_slots, self.head_dim))
            self.total_slots = self.active_slots = self.actual_slots
            if self.actual_slots != self.head_dim:
                self.slot_proj_k = nn.Linear(self.head_dim, self.actual_slots, bias=False)
                self.slot_proj_q = nn.Linear(self.head_dim, self.actual_slots, bias=False)
                nn.init.orthogonal_(self.slot_proj_k.weight)
                with torch.no_grad():
                    self.slot_proj_q.weight.copy_(self.slot_proj_k.weight)
        self.q_scale = nn.Parameter(torch.ones(num_heads))
        self.out_proj = nn.Linear(dim, dim, bias=False)
        self.norm = nn.LayerNorm(dim)
        if dynamic_decay:
            self.proj_alpha = nn.Linear(dim, num_heads, bias=True)
            rel = min(max((decay_init - 0.99) / 0.01, 1e-3), 0.999)
            nn.init.zeros_(self.proj_alpha.weight)
            nn.init.constant_(self.proj_alpha.bias, math.log(rel / (1.0 - rel)))
        else:
            self.proj_alpha = None
        self.decay = nn.Parameter(torch.full((1, num_heads, 1, 1), decay_init), requires_grad=False)
        self.beta_bias = nn.Parameter(torch.full((1, num_heads, 1, 1), 0.0))

    # ------------------------------------------------------------------ helpers
    def _fused_router(self) -> bool:
        return (self.top_k is not None and len(self.grid_dim) == 2 and not self.subspace_slicing)

    def _route_dense(self, k, q):
        """memory.py:219-238: factorized Kronecker or slot-projection routing."""
        if self.axes_proj_k is not None:
            wk = F.normalize(self.axes_proj_k[0](k), p=2, dim=-1)
            wq = self.axes_proj_q[0](q)
            for pk, pq in zip(self.axes_proj_k[1:], self.axes_proj_q[1:]):
                wk = (wk.unsqueeze(-1) * F.normalize(pk(k), p=2, dim=-1).unsqueeze(-2)).flatten(-2, -1)
                wq = (wq.unsqueeze(-1) * pq(q).unsqueeze(-2)).flatten(-2, -1)
            return wk, wq
        if self.slot_proj_k is not None:
            return F.normalize(self.slot_proj_k(k), p=2, dim=-1), self.slot_proj_q(q)
        return k, q

    def _route_sparse_torch(self, k, q):
        """Routing in torch (memory.py:240-289) for the shapes the fused router does not
        take (other axis counts, subspace slicing) and for training, where the router
        weights need gradients."""
        shp = k.shape[:-1]
        kf, qf = k.reshape(-1, k.shape[-1]), q.reshape(-1, q.shape[-1])
        n = len(self.grid_dim)
        ks = kf.chunk(n, dim=-1) if self.subspace_slicing else [kf] * n
        qs = qf.chunk(n, dim=-1) if self.subspace_slicing else [qf] * n
        wk = wq = idx = None
        for a, (pk, pq, ka, qa) in enumerate(zip(self.axes_proj_k, self.axes_proj_q, ks, qs)):
            val, ix = torch.topk(pk(ka), self.top_k, dim=-1)
            uk = F.normalize(val, p=2, dim=-1)
            uq = F.normalize(torch.gather(pq(qa), -1, ix), p=2, dim=-1)
            if a == 0:
                wk, wq, idx = uk, uq, ix
            else:
                wk = (wk.unsqueeze(-1) * uk.unsqueeze(-2)).flatten(-2, -1)
                wq = (wq.unsqueeze(-1) * uq.unsqueeze(-2)).flatten(-2, -1)
                idx = (idx.unsqueeze(-1) * self.grid_dim[a] + ix.unsqueeze(-2)).flatten(-2, -1)
        return wk.view(*shp, -1), wq.view(*shp, -1), idx.view(*shp, -1)

    def _project(self, x):
        """memory.py:428-444 (sequence) / :553-566 (step): q, k, v, beta and the decay."""
        d, H, Dh = self.d_model, self.num_heads, self.head_dim
        packed = self.proj_qkv_beta(x)
        q, k, v = packed[..., :3 * d].chunk(3, dim=-1)
        beta_raw = packed[..., 3 * d:]
        lead = x.shape[:-1]
        if x.dim() == 3:       # [b, t, d] -> [b, H, t, Dh]
            q = q.view(*lead, H, Dh).transpose(1, 2)
            k = F.normalize(k.view(*lead, H, Dh).transpose(1, 2), p=2, dim=-1)
            v = v.view(*lead, H, Dh).transpose(1, 2)
            beta = torch.sigmoid(beta_raw.view(*lead, H, 1).transpose(1, 2) + self.beta_bias)
            decay = ((0.99 + 0.01 * torch.sigmoid(self.proj_alpha(x))).transpose(1, 2)
                     if self.proj_alpha is not None else None)
        else:                  # [b, d] -> [b, H, Dh]
            q = q.view(-1, H, Dh)
            k = F.normalize(k.view(-1, H, Dh), p=2, dim=-1)
            v = v.view(-1, H, Dh)
            beta = torch.sigmoid(beta_raw.view(-1, H, 1) + self.beta_bias.view(1, H, 1))
            decay = (0.99 + 0.01 * torch.sigmoid(self.proj_alpha(x))) if self.proj_alpha is not None else None
        return q, k, v, beta, decay

    # ------------------------------------------------------------------ forward
    def forward(self, x: torch.Tensor, state: Optional[torch.Tensor] = None, seq_offset: int = 0,
                use_chunkwise: Optional[bool] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """x [b, t, d] -> (norm(out_proj(y)) [b, t, d], state).  ``seq_offset`` and
        ``use_chunkwise`` are accepted for API compatibility; the kernel choice is the
        library's."""
        if not x.is_cuda:
            raise RuntimeError("deltagrid_b200.DeltaGridLayer runs on CUDA tensors")
        b, t, d = x.shape
        H, Dh = self.num_heads, self.head_dim
        q, k, v, beta, decay_t = self._project(x)
        dt = q.dtype
        beta = beta.squeeze(-1).to(dt)
        decay = decay_t.to(dt).contiguous() if decay_t is not None else self.decay.to(dt).view(H)
        grad = torch.is_grad_enabled() and (x.requires_grad or (state is not None and state.requires_grad)
                                            or any(p.requires_grad for p in self.parameters()))

        if self.top_k is not None:
            if state is None:
                state = torch.zeros(b, H, self.total_slots, Dh, device=x.device, dtype=v.dtype)
            if not grad and self._fused_router():
                # routing + recurrence, the state updated in place
                routers_k = [p.weight for p in self.axes_proj_k]
                routers_q = [p.weight for p in self.axes_proj_q]
                y, state, _, _ = ext.pkm_fused_forward(k.contiguous(), q.contiguous(), v.contiguous(), beta.contiguous(),
                                                      routers_k, routers_q, self.q_scale, decay, state, top_k=self.top_k)
            else:
                wk, wq, idx = self._route_sparse_torch(k, q)
                wq = wq * self.q_scale.to(dt).view(1, H, 1, 1)
                args = (v.contiguous(), beta.contiguous(), wk.to(dt).contiguous(), wq.to(dt).contiguous(),
                        idx.to(torch.int64).contiguous(), decay)
                if grad:
                    y, state = _PkmRecurrence.apply(*args, state)
                else:
                    y, state, _ = ext.pkm_forward(*args, state, False)
        else:
            if not grad and self.slot_proj_k is not None and dense_route_covers(k, self.slot_proj_k.weight):
                # inference: the slot-routing kernel (projection, normalisation, q_scale)
                wk, wq = dense_route(k.to(dt), q.to(dt), self.slot_proj_k.weight, self.slot_proj_q.weight,
                                     self.q_scale)
            else:
                wk, wq = self._route_dense(k, q)
                wq = wq * self.q_scale.to(dt).view(1, H, 1, 1)
            s0 = state.to(dt) if state is not None else None
            args = (q.contiguous(), v.contiguous(), beta.contiguous(), wk.to(dt).contiguous(), wq.to(dt).contiguous(),
                    decay)
            if grad:
                y, state = _DenseRecurrence.apply(*args, s0)
            else:
                y, state, _, _ = ext.forward(args[0], args[1], args[1], *args[2:], s0, False)
        out = y.transpose(1, 2).reshape(b, t, d)
        return self.norm(self.out_proj(out)), state

    def step(self, x: torch.Tensor, state: Optional[torch.Tensor] = None,
             seq_offset: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
        """One token x [b, 1, d] (memory.py:544-638).  The PKM state is updated in place."""
        b, t, d = x.shape
        if t != 1:
            raise ValueError(f"step() expects sequence length 1, got {t}")
        H, Dh = self.num_heads, self.head_dim
        q, k, v, beta, decay_t = self._project(x.squeeze(1))
        dt = q.dtype
        beta = beta.squeeze(-1).to(dt)
        decay = decay_t.to(dt).contiguous() if decay_t is not None else self.decay.to(dt).view(H)
        if self.top_k is not None:
            if state is None:
                state = torch.zeros(b, H, self.total_slots, Dh, device=x.device, dtype=v.dtype)
            if self._fused_router():
                wk, wq, idx = pkm_route(k.unsqueeze(2).contiguous(), q.unsqueeze(2).contiguous(),
                                        [p.weight for p in self.axes_proj_k], [p.weight for p in self.axes_proj_q],
                                        self.top_k, self.q_scale)
                wk, wq, idx = wk.squeeze(2), wq.squeeze(2), idx.squeeze(2)
            else:
                wk, wq, idx = self._route_sparse_torch(k, q)
                wq = wq * self.q_scale.to(dt).view(1, H, 1)
            y, state = ext.pkm_step(v.contiguous(), beta.contiguous(), wk.to(dt).contiguous(), wq.to(dt).contiguous(),
                                    idx.to(torch.int64).contiguous(), decay, state)
        else:
            if state is None:
                state = torch.zeros(b, H, self.actual_slots, Dh, device=x.device, dtype=x.dtype)
            wk, wq = self._route_dense(k, q)
            wq = wq * self.q_scale.to(dt).view(1, H, 1)
            y, state = ext.step(q, k, v, beta, wk.to(dt), wq.to(dt), decay, state.to(dt))
        return self.norm(self.out_proj(y.reshape(b, d))).unsqueeze(1), state


SparseDeltaPKMLayer = DeltaGridLayer
