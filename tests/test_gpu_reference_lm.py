"""The reference's own DeltaGridLM (src/models/language_model.py, blocks and layers
unchanged, installed into baseline/_ref) run end to end twice: on the reference's
CUDA extension (built from its sources into oracle/_ref) and on this repository's
drop-in (deltagrid_b200.hsru_delta_cuda).  Everything but the recurrence is the
reference's torch code, so the two runs differ only in the kernels.

Checked: prefill logits and memory states (dense forward), decode logits (dense
step; both runs decode the reference run's greedy tokens), and, in fp32, every parameter gradient of a language-modelling loss
(dense forward with save_for_backward plus the analytic backward, through the
reference's _DeltaGridAutogradFunction).  Bars, max|a-b|/max|b|: 1e-4 in fp32; in
fp16 / bf16 5e-3 / 2e-2 (the two kernel sets round the same fp32 sums in a
different order, and the difference passes through LayerNorms and the LM head).
Skipped when baseline/_ref or oracle/_ref is absent.
"""
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_err
from oracle.build_ref_cuda import load_prebuilt
from reference_model import load_reference_package, use_backend

pytestmark = pytest.mark.gpu

REF_EXT = load_prebuilt() if torch.cuda.is_available() else None
DG = load_reference_package()
if torch.cuda.is_available():
    from deltagrid_b200 import hsru_delta_cuda as ours

need_both = pytest.mark.skipif(REF_EXT is None or DG is None,
                               reason="reference package (baseline/_ref) or reference extension (oracle/_ref) absent")
TOL = {torch.float32: 1e-4, torch.float16: 5e-3, torch.bfloat16: 2e-2}


def _np(t):
    return t.detach().double().cpu().numpy()


def _model(dtype, slots=128, dynamic=True, seed=0):
    torch.manual_seed(seed)
    m = DG.DeltaGridLM(vocab_size=1000, d_model=128, num_layers=2, num_heads=2, num_slots=slots,
                       dynamic_decay=dynamic)
    return m.cuda().to(dtype).eval()


def _prefill_and_decode(model, ids, steps, backend, tokens=None):
    """Prefill, then `steps` decode steps.  Without `tokens` the decode is greedy and the
    chosen tokens are returned; with `tokens` (a greedy run's choices) those are fed, so
    that two backends decode the same sequence: a near-tied argmax may otherwise pick a
    different token on one backend and every later logit then differs."""
    use_backend(backend)
    chosen = []
    with torch.no_grad():
        out = model(ids, return_state=True)
        logits, states = out.logits, out.state
        tok = logits[:, -1].argmax(-1, keepdim=True) if tokens is None else tokens[0]
        dec = []
        for i in range(steps):
            chosen.append(tok)
            lg, states = model.step(tok, states=states, seq_offset=ids.shape[1] + i)
            dec.append(lg)
            if tokens is None:
                tok = lg[:, -1].argmax(-1, keepdim=True)
            elif i + 1 < steps:
                tok = tokens[i + 1]
    torch.cuda.synchronize()
    mem = [s for s in _state_tensors(states)]
    return logits, torch.cat(dec, 1), mem, chosen


def _state_tensors(states):
    """The per-layer memory states (DeltaGridState.to_legacy(): (memory, conv indicator) pairs)."""
    return [mem for mem, _ in states.to_legacy() if isinstance(mem, torch.Tensor)]


@need_both
@pytest.mark.parametrize("dtype,slots,dynamic", [(torch.float32, 128, True), (torch.float16, 128, True),
                                                 (torch.bfloat16, 256, True), (torch.float32, 256, False)])
def test_reference_lm_prefill_and_decode(dtype, slots, dynamic):
    model = _model(dtype, slots, dynamic)
    ids = torch.randint(0, 1000, (4, 96), generator=torch.Generator().manual_seed(1)).cuda()
    lr, dr, mr, toks = _prefill_and_decode(model, ids, 6, REF_EXT)
    lo, do, mo, _ = _prefill_and_decode(model, ids, 6, ours, tokens=toks)
    tol = TOL[dtype]
    assert rel_err(_np(lo), _np(lr)) < tol
    assert rel_err(_np(do), _np(dr)) < tol
    assert len(mo) == len(mr) == 2
    for a, b in zip(mo, mr):
        assert rel_err(_np(a), _np(b)) < tol


@need_both
def test_reference_lm_training_gradients():
    model = _model(torch.float32, 128, True, seed=3).train()
    ids = torch.randint(0, 1000, (2, 80), generator=torch.Generator().manual_seed(2)).cuda()
    grads = []
    for backend in (REF_EXT, ours):
        use_backend(backend)
        model.zero_grad(set_to_none=True)
        logits = model(ids, return_state=False).logits
        loss = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), ids[:, 1:].reshape(-1))
        loss.backward()
        torch.cuda.synchronize()
        grads.append({n: p.grad.detach().clone() for n, p in model.named_parameters() if p.grad is not None})
    ref, got = grads
    assert ref.keys() == got.keys() and len(ref) > 10
    for name in ref:
        assert rel_err(_np(got[name]), _np(ref[name])) < 1e-4, name
