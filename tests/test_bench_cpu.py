"""bench.py's contract on the CPU: the reference arm's JSON line (one line,
the driver's keys, a config identical to the headline arm's, a bounded
sample whose ms_per_step is the measured sample step) and the headline
config's sharding figures for several world sizes."""
from __future__ import annotations

import json
import subprocess
import sys
import types

from conftest import REPO


def test_reference_arm_line_on_cpu():
    proc = subprocess.run(
        [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1",
         "--warmup", "0", "--no-secondary"],
        capture_output=True, text=True, timeout=600, cwd=REPO)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    # the step is the measured sample: 4 sequences through one layer
    layers = d["config"]["layers"]
    assert abs(d["value"] - 4 / (d["ms_per_step"] * 1e-3 * layers)) < 1e-6 * d["value"]
    bench = _bench()
    args = types.SimpleNamespace(workload="llama3_8b", batch=None, layers=None,
                                 sharding="balanced")
    assert d["config"] == json.loads(json.dumps(bench.decode_config(bench.make_workload(args),
                                                                    args, 1)))


def test_headline_config_sharding():
    bench = _bench()
    args = types.SimpleNamespace(workload="llama3_8b", batch=None, layers=None,
                                 sharding="balanced")
    full = bench.make_workload(args)
    total = float(full.lengths.sum())
    for world in (1, 2, 4, 8):
        c = bench.decode_config(full, args, world)
        assert c["batch"] == 256 and c["layers"] == 32
        assert abs(c["mean_rank_tokens"] * world - total) < 1e-6
        assert c["mean_rank_tokens"] <= c["max_rank_tokens"] <= 1.01 * c["mean_rank_tokens"]


def _bench():
    sys.argv = [sys.argv[0]]
    sys.path.insert(0, str(REPO))
    import bench
    return bench
