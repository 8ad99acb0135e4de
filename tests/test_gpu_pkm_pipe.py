"""Pipelined PKM kernel (rows fetched D steps ahead, hazards forwarded from shared
memory) against the CPU oracle.  dg_pkm_forward takes it for fp32 state (and
16-bit shapes the warp-specialised kernel does not cover) at T >= 64 with
16-byte-aligned inputs; here it is selected explicitly.  Saving gathered rows
runs the one-step kernel, which gives a second GPU reference on identical
inputs."""
import numpy as np
import pytest
import torch

from conftest import rel_err
from inputs import STORAGE, TOL, pkm_inputs, to_np32
from oracle import oracle as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from deltagrid_b200 import hsru_delta_cuda as ext


def _oracle(d, dtype):
    out, st = O.pkm_forward(to_np32(d["v"]), to_np32(d["beta"]), to_np32(d["wk"]), to_np32(d["wq"]),
                            d["idx"].numpy(), to_np32(d["decay"]), to_np32(d["state"]), STORAGE[dtype])
    return O.round_to(out, STORAGE[dtype]), st


def _gpu(d, save=False):
    # the pipelined kernel explicitly (the default choice for 16-bit state is the
    # warp-specialised kernel); saving rows always runs the one-step kernel
    g = {n: t.cuda() for n, t in d.items()}
    return ext.pkm_forward_algo(g["v"], g["beta"], g["wk"], g["wq"], g["idx"], g["decay"], g["state"], save,
                                1 if save else 2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("B,H,G,K", [(2, 2, 8, 4), (1, 4, 16, 8), (16, 8, 32, 8)])
def test_pipe_against_oracle(dtype, B, H, G, K):
    # (8, 4): 16 of 64 slots per step -> rows recur inside the prefetch window all the time
    d = pkm_inputs(B, H, 128, G, K, 64, dtype, dynamic=(G == 16), seed=G + K + B, s_init_scale=0.2)
    out, st, _ = _gpu(d)
    yo, so = _oracle(d, dtype)
    assert rel_err(out.float().cpu().numpy(), yo) < TOL[dtype]
    assert rel_err(st.float().cpu().numpy(), so) < TOL[dtype]


def test_pipe_matches_one_step_kernel():
    d = pkm_inputs(2, 3, 512, 16, 8, 64, torch.float16, dynamic=True, seed=5, s_init_scale=0.3)
    o1, s1, _ = _gpu(d)                 # pipelined
    o2, s2, _ = _gpu(d, save=True)      # one step at a time (saving rows)
    assert rel_err(o1.float().cpu().numpy(), o2.float().cpu().numpy()) < 1e-3
    assert rel_err(s1.float().cpu().numpy(), s2.float().cpu().numpy()) < 1e-3


def _slot_hash(x):
    return ((x * 2654435761) & 0xFFFFFFFF) >> 20


def test_pipe_table_overflow_falls_back_exactly():
    # every 4th step carries 9 slots whose hashes start in one 8-wide probe window:
    # the 9th insert overflows and the next steps reload rows synchronously
    total, A, T = 1 << 16, 16, 256
    bucket = {}
    for x in range(total):
        bucket.setdefault(_slot_hash(x), []).append(x)
    dense = [xs for h, xs in sorted(bucket.items()) if len(xs) >= 9]
    rs = np.random.RandomState(0)
    d = pkm_inputs(1, 2, T, 256, 4, 64, torch.float32, seed=9, s_init_scale=0.1)
    idx = d["idx"].clone()
    for h in range(2):
        for t in range(T):
            if t % 4 == 0:
                xs = dense[rs.randint(len(dense))][:9]
                rest = rs.choice(total, A, replace=False)
                rest = [x for x in rest if x not in xs][: A - 9]
                row = list(xs) + list(rest)
            else:
                row = list(rs.choice(total, A, replace=False))
            idx[0, h, t] = torch.tensor(row, dtype=torch.int64)
    d["idx"] = idx
    out, st, _ = _gpu(d)
    yo, so = _oracle(d, torch.float32)
    assert rel_err(out.cpu().numpy(), yo) < 1e-5
    assert rel_err(st.cpu().numpy(), so) < 1e-5
