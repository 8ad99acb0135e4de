"""bench.py on a B200 at reduced sizes: the contract line's keys, and finite output
checksums after the end-to-end leg (which carries the PKM state in place from piece to
piece, so anything non-finite it wrote would reach the verification step)."""
import json
import math
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("workload,extra", [
    ("cfg2", ["--batch", "2", "--seq", "512"]),
    ("cfg3", ["--batch", "1", "--seq", "2048"]),
    ("cfg4", ["--batch", "1", "--seq", "2048"]),
])
def test_bench_line_small(workload, extra):
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--workload", workload, "--steps", "3",
                        "--warmup", "3", "--no-workloads", "--no-cpu", *extra],
                       capture_output=True, text=True, timeout=900, cwd=REPO)
    assert r.returncode == 0, r.stderr[-3000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "roofline", "e2e",
                "gpu_launches", "clocks", "config"):
        assert key in line, key
    assert line["value"] > 0 and line["e2e"]["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] > 0 and line["e2e"]["d2h_bytes_per_step"] > 0
    assert line["gpu_launches"] >= line["steps"]
    assert 0 < line["roofline"]["frac"] < 1.5
    sums = [x for rank in line["verify"]["output_checksums_per_rank"] for x in rank]
    assert sums and all(math.isfinite(x) for x in sums), sums
