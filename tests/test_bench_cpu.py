"""bench.py on the CPU: the algorithmic-byte arithmetic behind every roofline figure,
the strong-scaling batch shards, and the --impl reference arm's JSON line (the
reference's own CPU engines; no GPU leg without a GPU)."""
import json
import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)

import bench  # noqa: E402


def test_algorithmic_bytes_match_the_per_head_token_figures():
    # dense cfg2: (2 Dh + 2 S) 2 B + 2 B (v, y, wk, wq, beta) per head-token, plus the final state
    b, f = bench._algorithmic(bench.WORKLOADS["cfg2"])
    ht = 32 * 16 * 4096
    assert b == ht * 2306 + 32 * 16 * 512 * 64 * 2 == 4869586944
    assert f == ht * 6.0 * 512 * 64
    # PKM cfg3 and cfg4: 64 rows in and out (16 KiB), v, y, beta, wk, wq, int64 idx
    for name in ("cfg3", "cfg4"):
        b, _ = bench._algorithmic(bench.WORKLOADS[name])
        w = bench.WORKLOADS[name]
        assert b == w["B"] * w["H"] * w["T"] * 17410
    # decode cfg5: a layer reads and writes the whole state
    b, _ = bench._algorithmic(bench.WORKLOADS["cfg5"])
    assert b == 12 * 256 * 12 * (2 * 256 * 64 * 2 + 2 * 256 * 2 + 2 * 64 * 2 + 2 * 2)


def test_roofline_fraction_is_bytes_over_time_over_peak():
    w = bench.WORKLOADS["cfg2"]
    r = bench._roofline(w, 2.0, None)
    hbm, _, _ = bench._peaks()
    assert r["bound"] == "hbm" and r["unit"] == "GB/s"
    assert r["achieved"] == pytest.approx(4869586944 / 2.0e-3 / 1e9)
    assert r["frac"] == pytest.approx(r["achieved"] / hbm)


def test_strong_scaling_shards_cover_the_batch_once():
    from deltagrid_b200.shard import shard_range
    for B, world in ((32, 1), (32, 2), (32, 8), (16, 8), (8, 8), (5, 2)):
        got = [shard_range(B, world, r) for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == B
        assert all(a[1] == b[0] for a, b in zip(got, got[1:]))


@pytest.mark.skipif(not os.path.exists(os.path.join(REPO, "oracle", "_ref", "libdg_ref_engine.so")),
                    reason="reference engine (oracle/_ref) not built")
def test_reference_arm_prints_the_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--workload", "cfg1",
                        "--steps", "1", "--warmup", "1"], capture_output=True, text=True, env=env, timeout=600,
                       cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["value"] > 0 and line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "reference" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert "engine_q16" in line["cpu_legs"]


@pytest.mark.parametrize("B", [1, 2, 4, 5, 8, 16, 32, 256])
def test_dense_e2e_pieces_cover_the_batch_once(B):
    w = dict(bench.WORKLOADS["cfg2"], B=B)
    b = bench.e2e_pieces(w)
    assert b[0][0] == 0 and b[-1][1] == B and all(x[1] == y[0] for x, y in zip(b, b[1:]))
    assert all(hi > lo for lo, hi in b)
    if B >= 16:       # small first and last pieces, the middle in four
        assert len(b) == 6 and b[0][1] - b[0][0] == B // 16 == b[-1][1] - b[-1][0]
    assert bench.e2e_pieces(w, 4) == ([(i * B // 4, (i + 1) * B // 4) for i in range(4)] if B % 4 == 0 else [(0, B)])


def test_pkm_e2e_pieces_and_launch_counts():
    for name in ("cfg3", "cfg4"):
        w = bench.WORKLOADS[name]
        b = bench.e2e_pieces(w)
        assert len(b) == 8 and b[-1][1] == w["T"] and all((hi - lo) % 8 == 0 for lo, hi in b)
        # four step pieces of pre-pass and recurrence when 8 SMs stay free, else one of each
        assert bench.launches_per_step(w, sms=148) == 8
        assert bench.launches_per_step(w, sms=128) == 2
    w = dict(bench.WORKLOADS["cfg3"], T=512)
    assert bench.launches_per_step(w, sms=148) == 2
    assert bench.launches_per_step(bench.WORKLOADS["cfg2"], sms=148) == 1
    assert bench.launches_per_step(bench.WORKLOADS["cfg5"], sms=148) == 12
