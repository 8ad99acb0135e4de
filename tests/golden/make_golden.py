"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run with ``DELTAGRID_REF`` set to the reference project's root (``oracle/refpath.py``) and where
``oracle/_ref/libdg_ref_engine.so`` has been built (``make -C oracle ref``):

    python tests/golden/make_golden.py

Sources of truth, per fixture:

* ``dense_*.npz``  -- the reference PyTorch layer's per-step loop
  (src/modules/memory.py:524-539), reached through ``DeltaGridLayer.forward`` on
  CPU with pieces shorter than 16 tokens (so the loop, not ``chunk_forward``,
  runs; memory.py:516) and the state carried between pieces.  ``out_proj`` and
  ``norm`` are replaced by identities so the layer returns y itself.
  The kernel-level inputs (v, beta, wk, wq, decay) are prepared here exactly as
  memory.py:432-444 and :491-492 do; the tests re-derive y from them, so a
  mismatch in that preparation would show up as a failing pin.
* ``pkm_*.npz``    -- the same layer in Sparse Delta-PKM mode: routing from
  ``DeltaGridLayer._route_sparse_pkm`` (memory.py:240-289) and the recurrence
  from the CPU loop of memory.py:466-487.
* ``router_*.npz`` -- ``_route_sparse_pkm`` on a 128x128 grid, top-8.
* ``engine_*.npz`` -- the reference C++ engine (fp32 and Q16.16), compiled from
  its own sources into oracle/_ref/, exporting per-step kernel inputs and y.

Everything is seeded; rerunning reproduces the committed files bit for bit on
the same torch version.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
from refpath import reference_root  # noqa: E402

REF = reference_root()
sys.path.insert(0, REF)
sys.path.insert(0, REPO)

from src.modules.memory import DeltaGridLayer  # noqa: E402  (reference package)
from oracle import oracle as O  # noqa: E402


def _prep(layer: DeltaGridLayer, x: torch.Tensor):
    """memory.py:432-444 -- q, k, v, beta, decay from x."""
    b, t, d = x.shape
    H, Dh = layer.num_heads, layer.head_dim
    packed = layer.proj_qkv_beta(x)
    qkv, beta_raw = packed[:, :, :3 * d], packed[:, :, 3 * d:]
    q, k, v = qkv.chunk(3, dim=-1)
    q = q.view(b, t, H, Dh).transpose(1, 2)
    k = F.normalize(k.view(b, t, H, Dh).transpose(1, 2), p=2, dim=-1)
    v = v.view(b, t, H, Dh).transpose(1, 2)
    beta = torch.sigmoid(beta_raw.view(b, t, H, 1).transpose(1, 2) + layer.beta_bias)
    if layer.proj_alpha is not None:
        decay = (0.99 + 0.01 * torch.sigmoid(layer.proj_alpha(x))).transpose(1, 2)
    else:
        decay = layer.decay.view(H)
    return q, k, v, beta.squeeze(-1), decay


def _identity_readout(layer: DeltaGridLayer) -> None:
    layer.out_proj = nn.Identity()
    layer.norm = nn.Identity()


def _run_pieces(layer, x, state, piece=15):
    """Reference forward in pieces < 16 tokens (per-step loop), state carried."""
    ys = []
    for s in range(0, x.shape[1], piece):
        y, state = layer(x[:, s:s + piece], state=state)
        ys.append(y)
    y = torch.cat(ys, dim=1)
    b, t, d = y.shape
    return y.view(b, t, layer.num_heads, layer.head_dim).transpose(1, 2), state


@torch.no_grad()
def make_dense(name, d_model, heads, slots, dynamic, decay_init, B, T, seed):
    torch.manual_seed(seed)
    layer = DeltaGridLayer(d_model=d_model, num_heads=heads, num_slots=slots,
                           dynamic_decay=dynamic, decay_init=decay_init).eval()
    with torch.no_grad():
        layer.q_scale.copy_(0.75 + 0.5 * torch.rand(heads))
        layer.beta_bias.normal_(0.0, 0.5)
        if layer.proj_alpha is not None:
            layer.proj_alpha.weight.normal_(0.0, 0.3)
    _identity_readout(layer)
    x = torch.randn(B, T, d_model)
    s0 = 0.1 * torch.randn(B, heads, layer.actual_slots, layer.head_dim)
    q, k, v, beta, decay = _prep(layer, x)
    wk, wq = layer._route_dense(k, q)
    wq = wq * layer.q_scale.view(1, heads, 1, 1)
    y, s_final = _run_pieces(layer, x, s0.clone())
    np.savez_compressed(os.path.join(HERE, name), v=v.numpy(), beta=beta.numpy(), wk=wk.numpy(),
                        wq=wq.numpy(), decay=decay.contiguous().numpy(), s_init=s0.numpy(),
                        y=y.contiguous().numpy(), s_final=s_final.numpy(),
                        dynamic=np.array(int(dynamic)))


@torch.no_grad()
def make_pkm(name, d_model, heads, grid, top_k, dynamic, B, T, seed):
    torch.manual_seed(seed)
    layer = DeltaGridLayer(d_model=d_model, num_heads=heads, grid_dim=grid, top_k=top_k,
                           dynamic_decay=dynamic).eval()
    with torch.no_grad():
        layer.q_scale.copy_(0.75 + 0.5 * torch.rand(heads))
        for pq in layer.axes_proj_q:          # decouple query routing from key routing
            pq.weight.normal_(0.0, 1.0 / np.sqrt(layer.head_dim))
        if layer.proj_alpha is not None:
            layer.proj_alpha.weight.normal_(0.0, 0.3)
    _identity_readout(layer)
    x = torch.randn(B, T, d_model)
    total = int(np.prod(grid))
    s0 = 0.1 * torch.randn(B, heads, total, layer.head_dim)
    q, k, v, beta, decay = _prep(layer, x)
    wk, wq, idx = layer._route_sparse_pkm(k, q)
    wq = wq * layer.q_scale.view(1, heads, 1, 1)
    y, s_final = _run_pieces(layer, x, s0.clone(), piece=x.shape[1])   # PKM CPU loop for any T
    np.savez_compressed(os.path.join(HERE, name), v=v.numpy(), beta=beta.numpy(), wk=wk.numpy(),
                        wq=wq.numpy(), idx=idx.numpy().astype(np.int64),
                        decay=decay.contiguous().numpy(), y=y.contiguous().numpy(),
                        s_final=s_final.numpy(),
                        s_init=s0.numpy(), k=k.numpy(), q=q.numpy(),
                        router_k0=layer.axes_proj_k[0].weight.numpy(),
                        router_k1=layer.axes_proj_k[1].weight.numpy(),
                        router_q0=layer.axes_proj_q[0].weight.numpy(),
                        router_q1=layer.axes_proj_q[1].weight.numpy(),
                        q_scale=layer.q_scale.numpy(), dynamic=np.array(int(dynamic)))


@torch.no_grad()
def make_router(name, grid, top_k, Dh, N, seed):
    torch.manual_seed(seed)
    heads = 1
    layer = DeltaGridLayer(d_model=Dh * heads, num_heads=heads, grid_dim=grid, top_k=top_k,
                           dynamic_decay=False).eval()
    for pk, pq in zip(layer.axes_proj_k, layer.axes_proj_q):   # the N(0, 1/Dh) routers of the configs
        pk.weight.normal_(0.0, 1.0 / np.sqrt(Dh))
        pq.weight.normal_(0.0, 1.0 / np.sqrt(Dh))
    k = F.normalize(torch.randn(1, heads, N, Dh), dim=-1)
    q = torch.randn(1, heads, N, Dh)
    wk, wq, idx = layer._route_sparse_pkm(k, q)
    np.savez_compressed(os.path.join(HERE, name), k=k.numpy(), q=q.numpy(), wk=wk.numpy(),
                        wq=wq.numpy(), idx=idx.numpy().astype(np.int64),
                        router_k0=layer.axes_proj_k[0].weight.numpy(),
                        router_k1=layer.axes_proj_k[1].weight.numpy(),
                        router_q0=layer.axes_proj_q[0].weight.numpy(),
                        router_q1=layer.axes_proj_q[1].weight.numpy())


def make_engine(name, fxp, mode, H, Dh, T, seed, **kw):
    run = O.ref_fxp_layer_run if fxp else O.ref_f32_layer_run
    e = run(mode, H, Dh, T, seed, **kw)
    if mode != 2:
        e.pop("idx")
    np.savez_compressed(os.path.join(HERE, name), mode=np.array(mode), H=np.array(H),
                        Dh=np.array(Dh), **e)


def main():
    make_dense("dense_static_f32.npz", d_model=128, heads=2, slots=None, dynamic=False,
               decay_init=0.999, B=1, T=40, seed=11)
    make_dense("dense_slotproj_dyn_f32.npz", d_model=64, heads=2, slots=128, dynamic=True,
               decay_init=0.995, B=1, T=24, seed=12)
    make_pkm("pkm_g16_k4_f32.npz", d_model=64, heads=2, grid=(16, 16), top_k=4, dynamic=True,
             B=1, T=24, seed=13)
    make_pkm("pkm_g32_k8_f32.npz", d_model=32, heads=1, grid=(32, 32), top_k=8, dynamic=False,
             B=1, T=16, seed=14)
    make_router("router_g128_k8.npz", grid=(128, 128), top_k=8, Dh=64, N=128, seed=15)
    make_engine("engine_f32_dense_dyn.npz", False, 0, H=2, Dh=32, T=12, seed=21, dyn=True)
    make_engine("engine_f32_pkm.npz", False, 2, H=2, Dh=32, T=12, seed=22, G0=16, G1=16, topk=4)
    make_engine("engine_fxp_dense_dyn.npz", True, 0, H=2, Dh=32, T=12, seed=23, dyn=True)
    make_engine("engine_fxp_slotproj.npz", True, 1, H=2, Dh=32, T=12, seed=24, slots=64)
    make_engine("engine_fxp_pkm.npz", True, 2, H=2, Dh=32, T=12, seed=25, G0=16, G1=16, topk=4)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f"{f}: {os.path.getsize(os.path.join(HERE, f))} bytes")


if __name__ == "__main__":
    main()
