"""Sharded execution on 2 CPU ranks over gloo: each rank runs its batch shard
(the CPU oracle stands in for the kernel), results gathered to rank 0 must equal
a single-process run.  Also: a rank that fails before the gather makes the
others' collective end with an error instead of hanging."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from deltagrid_b200.shard import checksum, gather_to_rank0, shard_range


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_range_covers_exactly():
    for n in (1, 5, 32, 33):
        for world in (1, 2, 3, 8):
            got = []
            for r in range(world):
                a, b = shard_range(n, world, r)
                got.extend(range(a, b))
            assert got == list(range(n))


def _worker(rank, world, port, result_path, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import oracle as O
    from tests.inputs import dense_inputs, to_np32
    d = dense_inputs(6, 2, 24, 64, 32, torch.float32, dynamic=True, seed=3)
    a, b = shard_range(6, world, rank)
    if rank == fail_rank:
        dist.destroy_process_group()
        raise SystemExit(3)
    try:
        out, s = O.dense_forward(*(to_np32(d[k][a:b]) for k in ("v", "beta", "wk", "wq", "decay")))
        ys = gather_to_rank0(torch.from_numpy(out))
        ss = gather_to_rank0(torch.from_numpy(s))
        cs = checksum(torch.from_numpy(out))
        all_cs = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(all_cs, cs)
        if rank == 0:
            np.savez(result_path, y=torch.cat(ys).numpy(), s=torch.cat(ss).numpy(),
                     cs=torch.stack(all_cs).numpy())
        status = 0
    except RuntimeError:
        status = 5
    dist.destroy_process_group()
    raise SystemExit(status)


def test_two_rank_shards_match_single_process(tmp_path):
    from oracle import oracle as O
    from inputs import dense_inputs, to_np32
    path = str(tmp_path / "r.npz")
    ctx = mp.get_context("spawn")
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, path, -1)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(120)
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    d = dense_inputs(6, 2, 24, 64, 32, torch.float32, dynamic=True, seed=3)
    out, s = O.dense_forward(*(to_np32(d[k]) for k in ("v", "beta", "wk", "wq", "decay")))
    r = np.load(path)
    np.testing.assert_array_equal(r["y"], out)
    np.testing.assert_array_equal(r["s"], s)
    full = checksum(torch.from_numpy(out[:3])).numpy()
    np.testing.assert_allclose(r["cs"][0], full, rtol=1e-12)


def test_failed_rank_ends_collective_with_error(tmp_path):
    path = str(tmp_path / "r.npz")
    ctx = mp.get_context("spawn")
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, path, 1)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(120)
    assert all(p.exitcode is not None for p in ps)     # nobody hangs
    assert ps[1].exitcode == 3
    assert ps[0].exitcode != 0                        # the survivor sees the failure
