"""dg_pkm_forward_noalloc, the entry point for callers that may not allocate device
memory while the recurrence runs (a serving loop with its memory reserved up front,
code under an allocator that forbids growth), checked against dg_pkm_forward, which
takes its scratch from the stream-ordered pool.  Identical inputs, two calls in a
row, so the second call reuses the fixed scratch array the first one filled and
both perform the per-device address look-up; over fp16 and bf16, static and per-step
decay, with and without the saved rows, and a call short enough to need no scratch.  Plus the size check:
a call needing more than the 16 MiB array is refused before any launch.  This file
is collected last so it also runs after every other GPU test in one process."""
import ctypes

import pytest
import torch

from inputs import pkm_inputs

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from deltagrid_b200 import _lib

F16, BF16 = 2, 3
CODE = {torch.float16: F16, torch.bfloat16: BF16}


def _args(g, B, H, T, A, total, status, dtype=torch.float16, dyn=0, saved=None):
    return (CODE[dtype], B, H, T, A, ctypes.c_int64(total), 64, g["v"].data_ptr(), g["beta"].data_ptr(),
            g["wk"].data_ptr(), g["wq"].data_ptr(), g["idx"].data_ptr(), g["decay"].data_ptr(), dyn,
            g["state"].data_ptr(), g["out"].data_ptr(), saved.data_ptr() if saved is not None else None,
            status.data_ptr(), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("B,H,G,T,dtype,dyn,save", [
    (16, 8, 32, 256, torch.float16, False, False),    # full rows
    (2, 3, 16, 256, torch.float16, False, False),     # row halves
    (2, 3, 16, 256, torch.bfloat16, True, False),     # bf16, per-step decay
    (2, 2, 32, 128, torch.float16, True, True),       # with the saved rows (save_for_backward)
    (2, 2, 32, 32, torch.float16, False, False),      # T < 64: a kernel without scratch, no array needed
])
def test_noalloc_matches_dg_pkm_forward_twice(B, H, G, T, dtype, dyn, save):
    K = 8
    d = pkm_inputs(B, H, T, G, K, 64, dtype, dynamic=dyn, seed=B + G + T, s_init_scale=0.2)
    runs = {}
    for name in ("dg_pkm_forward", "dg_pkm_forward_noalloc"):
        g = {n: t.cuda() for n, t in d.items()}
        g["out"] = torch.empty_like(g["v"])
        saved = torch.zeros(B, H, T, K * K, 64, dtype=dtype, device="cuda") if save else None
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        outs = []
        for _ in range(2):                       # second call continues from the first call's state
            _lib.call(name, *_args(g, B, H, T, K * K, G * G, status, dtype, int(dyn), saved))
            torch.cuda.synchronize()
            outs.append(g["out"].clone())
        assert int(status.item()) == 0
        runs[name] = (outs, g["state"].clone(), saved)
    (o1, s1, v1), (o2, s2, v2) = runs["dg_pkm_forward"], runs["dg_pkm_forward_noalloc"]
    for a, b in zip(o1, o2):
        assert torch.equal(a, b)
    assert torch.equal(s1, s2)
    if save:
        assert torch.equal(v1, v2)


def test_noalloc_rejects_oversize_without_launching():
    # 131080 steps of one lane need 131080 * 128 bytes > 16 MiB of scratch
    T = 131080
    g = {n: torch.zeros(16, dtype=torch.float16, device="cuda") for n in ("v", "beta", "wk", "wq", "decay", "state",
                                                                            "out")}
    g["idx"] = torch.zeros(16, dtype=torch.int64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib.lib().dg_pkm_forward_noalloc(*_args(g, 1, 1, T, 64, 1 << 14, status))
    assert rc == -4                                   # DG_ERR_WORKSPACE
